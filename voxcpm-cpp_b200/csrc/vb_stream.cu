// vb_stream.cu -- persistent weight-streaming GEMV programs.
//
// A batch-1 decode step is a chain of small dependent mat-muls (every
// ggml_mul_mat of src/minicpm4.c:270-458 at M=1).  Launched one by one, each
// pays launch latency, an activation prologue and a cold HBM pipeline, and
// the step ends up far below the bandwidth roofline.  This file runs a whole
// program of GEMVs in ONE cooperative launch with one CTA per SM:
//
//   warp 0 (producer)   walks the program in order and, for this CTA's slice
//                        of every weight, issues 1-D TMA bulk copies
//                        (cp.async.bulk, no multicast) of row chunks into a
//                        5-stage shared-memory ring, each stage completing
//                        an mbarrier by transaction bytes;
//   warps 1..8          quantize the activation of each op once into shared
//   (consumers)          memory (ggml's Q8_0 rule, bit-exact), then reduce
//                        every row chunk from the ring with dp4a block dots
//                        and write the outputs through the epilogue.
//
// Ops carry a dependency group: before reading its activation an op waits
// until every CTA has finished the group it depends on (a grid-wide
// counter).  The producer does not wait for dependencies -- weights do not
// depend on activations -- so it keeps HBM busy through the barriers, up to
// the ring depth.  Every wait is bounded: on timeout the kernel records an
// error code, stops issuing work, drains its own bulk copies and exits.
#include "vb_common.cuh"
#include "vb_kernels.cuh"
#include "vb_device.cuh"
#include "vb_stream.cuh"

namespace vb {

struct StreamOp {
    const uint8_t *w;       // Q8_0 qs int8 [N][K] or fp16 [N][K]
    const uint16_t *sc;     // Q8_0 scales fp16 [N][K/32]
    const float *x;
    float *y;
    const float *bias;
    int64_t ldx, ldy;
    int wtype, K, N, M;
    unsigned flags;
    int group, wait_group, last_in_group;
    int rows_per_chunk, row_bytes, sc_bulk;
};

constexpr int ST_STAGES = 5;
constexpr int ST_SLOT = 32768;                  // weight bytes per ring stage
constexpr int ST_SC_SLOT = ST_SLOT / 16;        // Q8_0 scale bytes per stage
constexpr int ST_CONSUMER_WARPS = 8;
constexpr int ST_CONSUMERS = ST_CONSUMER_WARPS * 32;
constexpr int ST_THREADS = ST_CONSUMERS + 32;
constexpr int ST_XBYTES = 16384;                // activation operand (int8 or fp16)
constexpr int ST_MMAX = 8;
constexpr size_t ST_SMEM = (size_t)ST_STAGES * ST_SLOT + (size_t)ST_STAGES * ST_SC_SLOT + ST_XBYTES +
                           (ST_XBYTES / 32) * 4 + 2 * ST_STAGES * 8 + 64;

__device__ __forceinline__ void stream_store(const StreamOp &op, int m, int64_t n, float v) {
    if (op.bias) v = __fadd_rn(v, op.bias[n]);
    if (op.flags & VB_OUT_BF16) v = bf16r(v);
    op.y[(int64_t)m * op.ldy + n] = v;
}

// Bounded wait on an mbarrier phase; false on timeout or abort.
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
    }
    return true;
}

__device__ __forceinline__ bool wait_grid(const unsigned *ctr, unsigned target, volatile int *abort_flag) {
    const long long t0 = clock64();
    while (ld_acquire_gpu(ctr) < target) {
        if (*abort_flag) return false;
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ void rows_of(int64_t N, int cta, int G, int64_t &r0, int64_t &r1) {
    r0 = N * cta / G;
    r1 = N * (cta + 1) / G;
}

__device__ __forceinline__ int dot32_i8(const int4 &a0, const int4 &a1, const int4 &b0, const int4 &b1) {
    // two independent dp4a chains, joined at the end (exact int32)
    int s0 = __dp4a(a0.x, b0.x, 0), s1 = __dp4a(a1.x, b1.x, 0);
    s0 = __dp4a(a0.y, b0.y, s0);
    s1 = __dp4a(a1.y, b1.y, s1);
    s0 = __dp4a(a0.z, b0.z, s0);
    s1 = __dp4a(a1.z, b1.z, s1);
    s0 = __dp4a(a0.w, b0.w, s0);
    s1 = __dp4a(a1.w, b1.w, s1);
    return s0 + s1;
}

// One ring chunk of a Q8_0 op: warp cw reduces rows 2cw, 2cw+1 (then +16,
// ...); each lane owns whole 32-value blocks, so one scale pair serves 32
// products.  y[m][n] = sum_b float(isum_b) * (d_w * d_x).  MC is the exact
// number of activation rows, so no predicated work is issued for absent rows.
template <int MC>
__device__ __forceinline__ void q8_chunk(const StreamOp &op, const uint8_t *__restrict__ wt,
                                         const uint16_t *__restrict__ sct, const int8_t *__restrict__ xq,
                                         const float *__restrict__ xd, int nr, int cw, int lane, int64_t r) {
    const int K = op.K, nb = K >> 5;
    for (int j0 = 2 * cw; j0 < nr; j0 += 2 * ST_CONSUMER_WARPS) {
        const bool two = (j0 + 1) < nr;
        const int8_t *w0 = reinterpret_cast<const int8_t *>(wt) + (int64_t)j0 * K;
        const int8_t *w1 = w0 + (two ? K : 0);
        float acc0[MC], acc1[MC];
#pragma unroll
        for (int m = 0; m < MC; m++) { acc0[m] = 0.0f; acc1[m] = 0.0f; }
#pragma unroll 2
        for (int b = lane; b < nb; b += 32) {
            const int4 a0 = *reinterpret_cast<const int4 *>(w0 + b * 32);
            const int4 a1 = *reinterpret_cast<const int4 *>(w0 + b * 32 + 16);
            const int4 c0 = *reinterpret_cast<const int4 *>(w1 + b * 32);
            const int4 c1 = *reinterpret_cast<const int4 *>(w1 + b * 32 + 16);
            const float s0 = h2f(sct[j0 * nb + b]);
            const float s1 = h2f(sct[(j0 + (two ? 1 : 0)) * nb + b]);
#pragma unroll
            for (int m = 0; m < MC; m++) {
                const int4 x0 = *reinterpret_cast<const int4 *>(xq + m * K + b * 32);
                const int4 x1 = *reinterpret_cast<const int4 *>(xq + m * K + b * 32 + 16);
                const float dx = xd[m * nb + b];
                acc0[m] = fmaf((float)dot32_i8(a0, a1, x0, x1), __fmul_rn(s0, dx), acc0[m]);
                acc1[m] = fmaf((float)dot32_i8(c0, c1, x0, x1), __fmul_rn(s1, dx), acc1[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < MC; m++) {
            const float v0 = warp_sum(acc0[m]);
            const float v1 = warp_sum(acc1[m]);
            if (lane == 0) {
                stream_store(op, m, r + j0, v0);
                if (two) stream_store(op, m, r + j0 + 1, v1);
            }
        }
    }
}

// One ring chunk of an F16 op: lanes own 16-value (32-byte) pieces of a row,
// fp16 x fp16 products accumulated in fp32.
template <int MC>
__device__ __forceinline__ void f16_chunk(const StreamOp &op, const uint8_t *__restrict__ wt,
                                          const uint16_t *__restrict__ xh, int nr, int cw, int lane, int64_t r) {
    const int K = op.K, np = K >> 4;
    for (int j0 = 2 * cw; j0 < nr; j0 += 2 * ST_CONSUMER_WARPS) {
        const bool two = (j0 + 1) < nr;
        const uint8_t *w0 = wt + (int64_t)j0 * K * 2;
        const uint8_t *w1 = w0 + (two ? K * 2 : 0);
        float acc0[MC], acc1[MC];
#pragma unroll
        for (int m = 0; m < MC; m++) { acc0[m] = 0.0f; acc1[m] = 0.0f; }
#pragma unroll 2
        for (int p = lane; p < np; p += 32) {
            const int4 a0 = *reinterpret_cast<const int4 *>(w0 + p * 32);
            const int4 a1 = *reinterpret_cast<const int4 *>(w0 + p * 32 + 16);
            const int4 c0 = *reinterpret_cast<const int4 *>(w1 + p * 32);
            const int4 c1 = *reinterpret_cast<const int4 *>(w1 + p * 32 + 16);
#pragma unroll
            for (int m = 0; m < MC; m++) {
                const int4 x0 = *reinterpret_cast<const int4 *>(xh + m * K + p * 16);
                const int4 x1 = *reinterpret_cast<const int4 *>(xh + m * K + p * 16 + 8);
                acc0[m] = dot8_f16(a1, x1, dot8_f16(a0, x0, acc0[m]));
                acc1[m] = dot8_f16(c1, x1, dot8_f16(c0, x0, acc1[m]));
            }
        }
        if ((K & 15) && lane == 0) {   // tail of 8 values (K a multiple of 8, not 16)
            const int4 a0 = *reinterpret_cast<const int4 *>(w0 + np * 32);
            const int4 c0 = *reinterpret_cast<const int4 *>(w1 + np * 32);
#pragma unroll
            for (int m = 0; m < MC; m++) {
                const int4 x0 = *reinterpret_cast<const int4 *>(xh + m * K + np * 16);
                acc0[m] = dot8_f16(a0, x0, acc0[m]);
                acc1[m] = dot8_f16(c0, x0, acc1[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < MC; m++) {
            const float v0 = warp_sum(acc0[m]);
            const float v1 = warp_sum(acc1[m]);
            if (lane == 0) {
                stream_store(op, m, r + j0, v0);
                if (two) stream_store(op, m, r + j0 + 1, v1);
            }
        }
    }
}

// Decode fast path (Q8_0, M = 1): LPR lanes own one weight row, lane s of a
// row handles the 16-byte half-blocks s, s+LPR, ..., so every quarter-warp
// reads 128 contiguous shared-memory bytes (no bank conflicts).  The lane's
// slice of the quantized activation (IT half-blocks) and its scales stay in
// registers for the whole op, so shared memory carries only the weights.
// Each half-block contributes float(isum_16) * (d_w * d_x); a row is reduced
// over its LPR lanes.  Returns false on a timeout or an abort.
template <int LPR, int IT>
__device__ __forceinline__ bool q8_m1_op(const StreamOp &op, const uint8_t *wslot, const uint8_t *sslot,
                                         const int8_t *xq, const float *xd, uint64_t *full, uint64_t *empty,
                                         int &slot, uint32_t &phase, int64_t r0, int64_t r1, int cw, int lane,
                                         volatile int *abort_flag, int *err) {
    constexpr int RPW = 32 / LPR;                       // rows per warp per pass
    constexpr int RPP = RPW * ST_CONSUMER_WARPS;        // rows per pass of all warps
    const int K = op.K, nb = K >> 5;
    const int ls = lane % LPR, lr = lane / LPR;
    int4 xr[IT];
    float dxr[IT];
#pragma unroll
    for (int i = 0; i < IT; i++) {
        const int hb = ls + LPR * i;
        xr[i] = *reinterpret_cast<const int4 *>(xq + hb * 16);
        dxr[i] = xd[hb >> 1];
    }
    float *y = op.y;
    const float *bias = op.bias;
    const bool b16 = op.flags & VB_OUT_BF16;
    const int R = op.rows_per_chunk;
    const bool sc_bulk = op.sc_bulk != 0;
    const uint16_t *scg = op.sc;
    for (int64_t r = r0; r < r1; r += R) {
        const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
        if (!wait_phase(&full[slot], phase, abort_flag)) {
            if (!*abort_flag) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); *abort_flag = 1; }
            return false;
        }
        const int8_t *wt = reinterpret_cast<const int8_t *>(wslot + (size_t)slot * ST_SLOT);
        const uint16_t *sct = sc_bulk ? reinterpret_cast<const uint16_t *>(sslot + (size_t)slot * ST_SC_SLOT)
                                      : scg + r * nb;
        for (int jb = cw * RPW; jb < nr; jb += RPP) {   // warp-uniform
            const int j = jb + lr;
            const bool valid = j < nr;
            const int jj = valid ? j : jb;
            const int8_t *wr = wt + (int64_t)jj * K;
            const uint16_t *sr = sct + jj * nb;
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < IT; i++) {
                const int hb = ls + LPR * i;
                const int4 wv = *reinterpret_cast<const int4 *>(wr + hb * 16);
                const float s = __fmul_rn(h2f(sr[hb >> 1]), dxr[i]);
                acc = fmaf((float)dot16_i8(wv, xr[i]), s, acc);
            }
#pragma unroll
            for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (valid && ls == 0) {
                float v = acc;
                const int64_t n = r + j;
                if (bias) v = __fadd_rn(v, bias[n]);
                if (b16) v = bf16r(v);
                y[n] = v;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == ST_STAGES) { slot = 0; phase ^= 1u; }
    }
    return true;
}

__global__ void __launch_bounds__(ST_THREADS, 1)
    stream_gemv_kernel(const StreamOp *__restrict__ ops, int n_ops, unsigned *bars, int *err) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t *wslot = sm;
    uint8_t *sslot = wslot + (size_t)ST_STAGES * ST_SLOT;
    int8_t *xq = reinterpret_cast<int8_t *>(sslot + (size_t)ST_STAGES * ST_SC_SLOT);
    float *xd = reinterpret_cast<float *>(xq + ST_XBYTES);
    uint64_t *full = reinterpret_cast<uint64_t *>(xd + ST_XBYTES / 32);
    uint64_t *empty = full + ST_STAGES;
    __shared__ volatile int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ST_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ST_CONSUMER_WARPS);
        }
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();

    // ------------------------------------------------------------ producer
    if (warp == 0) {
        if (lane != 0) return;
        int slot = 0;
        uint32_t phase = 0;
        long long fills = 0;
        for (int i = 0; i < n_ops && !s_abort; i++) {
            const StreamOp &op = ops[i];
            int64_t r0, r1;
            rows_of(op.N, cta, G, r0, r1);
            const int R = op.rows_per_chunk;
            const int nb = op.K / QK;
            for (int64_t r = r0; r < r1; r += R) {
                const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
                if (!wait_phase(&empty[slot], phase ^ 1u, &s_abort)) {
                    if (!s_abort) { atomicCAS(err, 0, STREAM_TIMEOUT_EMPTY); s_abort = 1; }
                    break;
                }
                const uint32_t wb = (uint32_t)nr * (uint32_t)op.row_bytes;
                const uint32_t sb = op.sc_bulk ? (uint32_t)nr * (uint32_t)nb * 2u : 0u;
                mbar_arrive_expect_tx(&full[slot], wb + sb);
                bulk_g2s(wslot + (size_t)slot * ST_SLOT, op.w + r * op.row_bytes, wb, &full[slot]);
                if (sb) bulk_g2s(sslot + (size_t)slot * ST_SC_SLOT, op.sc + r * nb, sb, &full[slot]);
                fills++;
                if (++slot == ST_STAGES) { slot = 0; phase ^= 1u; }
            }
        }
        // Drain: the last fill of every stage must have landed before this
        // thread exits (normally the consumers have already seen it).
        for (int s = 0; s < ST_STAGES; s++) {
            const long long n_s = fills / ST_STAGES + ((fills % ST_STAGES) > s ? 1 : 0);
            if (n_s == 0) continue;
            const uint32_t par = (uint32_t)((n_s - 1) & 1);
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], par)) {
                if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); break; }
            }
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int ctid = threadIdx.x - 32, cw = warp - 1;
    int slot = 0;
    uint32_t phase = 0;
    const float *last_x = nullptr;
    int last_K = -1, last_M = -1, last_type = -1;
    int64_t last_ldx = -1;
    int waited = -1;    // highest group this CTA has already waited for
    bool bad = false;   // this thread saw a timeout or an abort
    // Every consumer_sync / consumer_sync_or below is executed by all
    // consumer warps in the same order; loops end only on a uniform flag.
    for (int i = 0; i < n_ops; i++) {
        const StreamOp &op = ops[i];
        if (op.wait_group > waited) {
            if (ctid == 0 && !wait_grid(bars + op.wait_group, (unsigned)G, &s_abort)) {
                if (!s_abort) { atomicCAS(err, 0, STREAM_TIMEOUT_GRID); s_abort = 1; }
                bad = true;
            }
            if (consumer_sync_or(bad || s_abort, ST_CONSUMERS)) break;
            waited = op.wait_group;
            last_x = nullptr;   // the activation may have been rewritten
        }
        const int K = op.K, M = op.M, nb = K / QK;
        int64_t r0, r1;
        rows_of(op.N, cta, G, r0, r1);
        // The previous op ended with a consumer barrier, so no warp still
        // reads the activation buffers when they are rewritten here.
        if (r1 > r0 &&
            !(op.x == last_x && K == last_K && M == last_M && op.wtype == last_type && op.ldx == last_ldx)) {
            if (op.wtype == VB_TYPE_Q8_0) {
                // four threads per 32-value block (8 values each), ggml's
                // rule, bit-exact: amax over the block, d = amax/127 (fp16),
                // q = round-half-even(x * 127/amax)
                const int total = M * nb * 4;
                for (int base = 0; base < total; base += ST_CONSUMERS) {
                    const int item = base + ctid;
                    const bool valid = item < total;
                    const int blk = valid ? (item >> 2) : 0, part = item & 3;
                    const int m = blk / nb, kb = blk % nb;
                    float v[8];
                    if (valid) {
                        const float4 *src =
                            reinterpret_cast<const float4 *>(op.x + (int64_t)m * op.ldx + kb * QK + part * 8);
                        const float4 f0 = __ldcg(src), f1 = __ldcg(src + 1);
                        v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
                        v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; e++) v[e] = 0.0f;
                    }
                    float amax = 0.0f;
#pragma unroll
                    for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(v[e]));
                    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                    const float d = __fdiv_rn(amax, 127.0f);
                    const uint16_t dh = f2h(d);
                    const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
                    uint32_t pk[2];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        uint32_t w4 = 0;
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int q = __float2int_rn(__fmul_rn(v[4 * h + e], id));
                            w4 |= ((uint32_t)(q & 0xff)) << (8 * e);
                        }
                        pk[h] = w4;
                    }
                    if (valid) {
                        *reinterpret_cast<uint2 *>(xq + (int64_t)m * K + kb * QK + part * 8) = make_uint2(pk[0], pk[1]);
                        if (part == 0) xd[m * nb + kb] = h2f(dh);
                    }
                }
            } else {
                // fp16 operand, 8 values per thread
                uint16_t *xh = reinterpret_cast<uint16_t *>(xq);
                const int total = M * K / 8;
                for (int e = ctid; e < total; e += ST_CONSUMERS) {
                    const int m = (e * 8) / K, k = (e * 8) % K;
                    const float4 *src = reinterpret_cast<const float4 *>(op.x + (int64_t)m * op.ldx + k);
                    const float4 f0 = __ldcg(src), f1 = __ldcg(src + 1);
                    uint4 o;
                    o.x = (uint32_t)f2h(f0.x) | ((uint32_t)f2h(f0.y) << 16);
                    o.y = (uint32_t)f2h(f0.z) | ((uint32_t)f2h(f0.w) << 16);
                    o.z = (uint32_t)f2h(f1.x) | ((uint32_t)f2h(f1.y) << 16);
                    o.w = (uint32_t)f2h(f1.z) | ((uint32_t)f2h(f1.w) << 16);
                    *reinterpret_cast<uint4 *>(xh + (int64_t)m * K + k) = o;
                }
            }
            consumer_sync(ST_CONSUMERS);
            last_x = op.x;
            last_K = K;
            last_M = M;
            last_type = op.wtype;
            last_ldx = op.ldx;
        }

        bool fast_done = false;
        if (op.wtype == VB_TYPE_Q8_0 && M == 1) {
            bool ok = true;
            fast_done = true;
            switch (K) {
                case 1024: ok = q8_m1_op<16, 4>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err); break;
                case 2048: ok = q8_m1_op<16, 8>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err); break;
                case 4096: ok = q8_m1_op<16, 16>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err); break;
                case 6144: ok = q8_m1_op<32, 12>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err); break;
                case 8192: ok = q8_m1_op<32, 16>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err); break;
                default: fast_done = false; break;
            }
            if (!ok) bad = true;
        }
        const int R = op.rows_per_chunk;
        for (int64_t r = r0; !fast_done && r < r1; r += R) {
            const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
            if (!wait_phase(&full[slot], phase, &s_abort)) {
                if (!s_abort) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); s_abort = 1; }
                bad = true;
                break;
            }
            const uint8_t *wt = wslot + (size_t)slot * ST_SLOT;
            if (op.wtype == VB_TYPE_Q8_0) {
                const uint16_t *sct = op.sc_bulk ? reinterpret_cast<const uint16_t *>(sslot + (size_t)slot * ST_SC_SLOT)
                                                 : op.sc + r * nb;
                switch (M) {
                    case 1: q8_chunk<1>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 2: q8_chunk<2>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 3: q8_chunk<3>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 4: q8_chunk<4>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 5: q8_chunk<5>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 6: q8_chunk<6>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 7: q8_chunk<7>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    default: q8_chunk<8>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                }
            } else {
                const uint16_t *xh = reinterpret_cast<const uint16_t *>(xq);
                switch (M) {
                    case 1: f16_chunk<1>(op, wt, xh, nr, cw, lane, r); break;
                    case 2: f16_chunk<2>(op, wt, xh, nr, cw, lane, r); break;
                    case 3: f16_chunk<3>(op, wt, xh, nr, cw, lane, r); break;
                    case 4: f16_chunk<4>(op, wt, xh, nr, cw, lane, r); break;
                    case 5: f16_chunk<5>(op, wt, xh, nr, cw, lane, r); break;
                    case 6: f16_chunk<6>(op, wt, xh, nr, cw, lane, r); break;
                    case 7: f16_chunk<7>(op, wt, xh, nr, cw, lane, r); break;
                    default: f16_chunk<8>(op, wt, xh, nr, cw, lane, r); break;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == ST_STAGES) { slot = 0; phase ^= 1u; }
        }
        if (consumer_sync_or(bad, ST_CONSUMERS)) break;
        if (op.last_in_group && ctid == 0) {
            __threadfence();
            red_release_gpu(bars + op.group, 1u);
        }
    }
}

}  // namespace vb

using namespace vb;

struct vb_program_s {
    StreamOp *d_ops = nullptr;
    unsigned *d_bars = nullptr;
    int *d_err = nullptr;
    int n_ops = 0, n_groups = 0, grid = 0;
    size_t weight_bytes = 0;
};

namespace vb {
int init_stream(vb_ctx *ctx) {
    VB_CHECK(ctx, cudaFuncSetAttribute(stream_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ST_SMEM));
    return VB_OK;
}
}  // namespace vb

extern "C" int vb_program_create(vb_ctx *ctx, int n_ops, const vb_gemv_op *ops, vb_program *out) {
    if (!ctx || n_ops <= 0 || !ops || !out) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    std::vector<StreamOp> h(n_ops);
    int n_groups = 0;
    size_t wbytes = 0;
    for (int i = 0; i < n_ops; i++) {
        const vb_gemv_op &o = ops[i];
        StreamOp &s = h[i];
        vb_weight w = o.w;
        if (!w || !o.x || !o.y || o.M < 1 || o.M > ST_MMAX)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: null pointer or M outside 1..%d", i, ST_MMAX);
        if (w->type != VB_TYPE_Q8_0 && w->type != VB_TYPE_F16)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: weight type must be Q8_0 or F16", i);
        if (o.group < 0 || (i > 0 && o.group < ops[i - 1].group) || o.wait_group >= o.group)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: groups must be non-decreasing and wait on an earlier group", i);
        if (i > 0 && o.group != ops[i - 1].group && o.group != ops[i - 1].group + 1)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: group ids must be consecutive", i);
        const int K = (int)w->K;
        s.wtype = w->type;
        s.K = K;
        s.N = (int)w->N;
        s.M = o.M;
        s.w = (const uint8_t *)w->data;
        s.sc = w->scales;
        s.x = o.x;
        s.y = o.y;
        s.bias = o.bias;
        s.ldx = o.ldx ? o.ldx : K;
        s.ldy = o.ldy ? o.ldy : w->N;
        s.flags = o.flags;
        s.group = o.group;
        s.wait_group = o.wait_group;
        s.last_in_group = (i == n_ops - 1) || (ops[i + 1].group != o.group);
        s.row_bytes = w->type == VB_TYPE_Q8_0 ? K : 2 * K;
        s.rows_per_chunk = ST_SLOT / s.row_bytes;
        s.sc_bulk = (w->type == VB_TYPE_Q8_0) && (K % 256 == 0);
        if (s.rows_per_chunk < 1 || s.row_bytes % 16)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: K=%d not supported by the streaming kernel", i, K);
        const int xbytes = (w->type == VB_TYPE_Q8_0 ? 1 : 2) * K * o.M;
        if (xbytes > ST_XBYTES)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: M*K operand exceeds %d bytes", i, ST_XBYTES);
        if (((uintptr_t)o.x & 15) || (s.ldx & 3))
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: x rows must be 16-byte aligned", i);
        n_groups = o.group + 1;
        wbytes += w->device_bytes;
    }
    int per_sm = 0;
    VB_CHECK(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stream_gemv_kernel, ST_THREADS, ST_SMEM));
    if (per_sm < 1) return set_error(ctx, VB_ERR_BACKEND, "streaming kernel does not fit on an SM");
    vb_program p = new vb_program_s();
    p->n_ops = n_ops;
    p->n_groups = n_groups;
    p->grid = ctx->sm_count;
    p->weight_bytes = wbytes;
    cudaError_t e = cudaMalloc(&p->d_ops, sizeof(StreamOp) * n_ops);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_bars, sizeof(unsigned) * n_groups);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpy(p->d_ops, h.data(), sizeof(StreamOp) * n_ops, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(p->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        vb_program_destroy(p);
        return check_cuda(ctx, e, "vb_program_create");
    }
    *out = p;
    return VB_OK;
}

extern "C" int vb_program_run(vb_ctx *ctx, vb_program p) {
    if (!ctx || !p) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaMemsetAsync(p->d_bars, 0, sizeof(unsigned) * p->n_groups, ctx->stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(ST_THREADS);
    cfg.dynamicSmemBytes = ST_SMEM;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VB_CHECK(ctx, cudaLaunchKernelEx(&cfg, stream_gemv_kernel, (const StreamOp *)p->d_ops, p->n_ops, p->d_bars,
                                     p->d_err));
    VB_LAUNCH_CHECK(ctx, "stream_gemv");
    return VB_OK;
}

extern "C" int vb_program_status(vb_ctx *ctx, vb_program p, int *device_error) {
    if (!ctx || !p || !device_error) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
    VB_CHECK(ctx, cudaMemcpy(device_error, p->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (*device_error) return set_error(ctx, VB_ERR_BACKEND, "streaming kernel reported error %d", *device_error);
    return VB_OK;
}

extern "C" void vb_program_destroy(vb_program p) {
    if (!p) return;
    cudaFree(p->d_ops);
    cudaFree(p->d_bars);
    cudaFree(p->d_err);
    delete p;
}
