// vb_stream_dev.cuh -- device side of the persistent streaming kernel:
// the op descriptor, ring geometry, bounded waits and the per-chunk
// mat-vec routines shared by GEMV programs and the decode step.
#pragma once

#include "vb_common.cuh"
#include "vb_device.cuh"
#include "vb_stream.cuh"
#include "vb_stream_op.cuh"

namespace vb {

// Cycles a wait on other CTAs (a grid dependency) may take before the kernel
// records a timeout: the launch argument of vb_set_wait_limit, per CTA.
__shared__ long long s_dep_limit;

// Output / input row of logical row m (identity unless the op carries a
// vb_matmul row mapping).
__device__ __forceinline__ int64_t out_row(const StreamOp &op, int m) {
    return op.seg > 0 ? (m / op.seg) * op.seg_stride + op.seg_off + m % op.seg : m;
}
__device__ __forceinline__ int64_t in_row(const StreamOp &op, int m) { return op.x_mod > 0 ? m % op.x_mod : m; }

// Epilogue of one output value: bias, the bf16 flag, then the block residual
// y = bf16(res + scale * value).  Values written earlier in the same launch
// (the residual stream) are read through L2 (__ldcg), never through the
// non-coherent per-SM L1.
__device__ __forceinline__ float stream_epilogue(const StreamOp &op, int m, int64_t n, float v) {
    if (op.bias) v = __fadd_rn(v, op.bias[n]);
    if (op.flags & VB_OUT_BF16) v = bf16r(v);
    if (op.epi == EPI_RESIDUAL) {
        if (op.res_scale != 1.0f) v = __fmul_rn(v, op.res_scale);
        return bf16r(__fadd_rn(__ldcg(op.res + out_row(op, m) * op.ldy + n), v));
    }
    return v;
}

// The same epilogue with the residual value already at hand.
__device__ __forceinline__ float stream_epilogue_res(const StreamOp &op, int64_t n, float v, float res) {
    if (op.bias) v = __fadd_rn(v, op.bias[n]);
    if (op.flags & VB_OUT_BF16) v = bf16r(v);
    if (op.res_scale != 1.0f) v = __fmul_rn(v, op.res_scale);
    return bf16r(__fadd_rn(res, v));
}

__device__ __forceinline__ void stream_store(const StreamOp &op, int m, int64_t n, float v) {
    op.y[out_row(op, m) * op.ldy + n] = stream_epilogue(op, m, n, v);
}

// Slot row of logical row j in a chunk of nr rows.  An EPI_SWIGLU chunk
// holds its gate rows then its up rows; logical rows interleave them
// (2t = gate t, 2t+1 = up t) so a pair is reduced by neighbouring lanes.
__device__ __forceinline__ int slot_row(int j, int nr, bool swz) {
    return swz ? ((j & 1) ? (nr >> 1) + (j >> 1) : (j >> 1)) : j;
}

__device__ __forceinline__ void swiglu_store(const StreamOp &op, int m, int64_t t, float g, float u) {
    op.y[out_row(op, m) * op.ldy + t] = bf16r(__fmul_rn(bf16r(silu_f(bf16r(g))), bf16r(u)));
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
        if (clock64() - t0 > s_dep_limit) return false;
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
    const bool swz = op.epi == EPI_SWIGLU;
    for (int j0 = 2 * cw; j0 < nr; j0 += 2 * ST_CONSUMER_WARPS) {
        const bool two = (j0 + 1) < nr;
        const int s0r = slot_row(j0, nr, swz), s1r = slot_row(j0 + (two ? 1 : 0), nr, swz);
        const int8_t *w0 = reinterpret_cast<const int8_t *>(wt) + (int64_t)s0r * K;
        const int8_t *w1 = reinterpret_cast<const int8_t *>(wt) + (int64_t)s1r * K;
        float acc0[MC], acc1[MC];
#pragma unroll
        for (int m = 0; m < MC; m++) { acc0[m] = 0.0f; acc1[m] = 0.0f; }
#pragma unroll 2
        for (int b = lane; b < nb; b += 32) {
            const int4 a0 = *reinterpret_cast<const int4 *>(w0 + b * 32);
            const int4 a1 = *reinterpret_cast<const int4 *>(w0 + b * 32 + 16);
            const int4 c0 = *reinterpret_cast<const int4 *>(w1 + b * 32);
            const int4 c1 = *reinterpret_cast<const int4 *>(w1 + b * 32 + 16);
            const float s0 = h2f(sct[s0r * nb + b]);
            const float s1 = h2f(sct[s1r * nb + b]);
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
                if (swz) {
                    swiglu_store(op, m, (r + j0) >> 1, v0, v1);
                } else {
                    stream_store(op, m, r + j0, v0);
                    if (two) stream_store(op, m, r + j0 + 1, v1);
                }
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
    const bool swz = op.epi == EPI_SWIGLU;
    for (int j0 = 2 * cw; j0 < nr; j0 += 2 * ST_CONSUMER_WARPS) {
        const bool two = (j0 + 1) < nr;
        const uint8_t *w0 = wt + (int64_t)slot_row(j0, nr, swz) * K * 2;
        const uint8_t *w1 = wt + (int64_t)slot_row(j0 + (two ? 1 : 0), nr, swz) * K * 2;
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
                if (swz) {
                    swiglu_store(op, m, (r + j0) >> 1, v0, v1);
                } else {
                    stream_store(op, m, r + j0, v0);
                    if (two) stream_store(op, m, r + j0 + 1, v1);
                }
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
// over its LPR lanes.  sres (optional) holds the residual rows r0 .. r1 of an
// EPI_RESIDUAL op, fetched ahead.  Returns false on a timeout or an abort.
template <int LPR, int IT>
__device__ __forceinline__ bool q8_m1_op(const StreamOp &op, const uint8_t *wslot, const uint8_t *sslot,
                                         const int8_t *xq, const float *xd, uint64_t *full, uint64_t *empty,
                                         int &slot, uint32_t &phase, int64_t r0, int64_t r1, int cw, int lane,
                                         volatile int *abort_flag, int *err, int ns, const float *sres = nullptr) {
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
    float *y = op.y + out_row(op, 0) * op.ldy;
    const float *bias = op.bias;
    const bool b16 = op.flags & VB_OUT_BF16;
    const bool residual = op.epi == EPI_RESIDUAL;
    const bool swz = op.epi == EPI_SWIGLU;   // needs RPW even (LPR <= 16)
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
            const int sj = slot_row(jj, nr, swz);
            const int8_t *wr = wt + (int64_t)sj * K;
            const uint16_t *sr = sct + sj * nb;
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
            if (swz) {
                const float up = __shfl_down_sync(0xffffffffu, acc, LPR);   // row j + 1
                if (valid && ls == 0 && !(lr & 1)) swiglu_store(op, 0, (r + j) >> 1, acc, up);
            } else if (valid && ls == 0) {
                const int64_t n = r + j;
                if (residual) {
                    y[n] = sres ? stream_epilogue_res(op, n, acc, sres[n - r0]) : stream_epilogue(op, 0, n, acc);
                } else {
                    float v = acc;
                    if (bias) v = __fadd_rn(v, bias[n]);
                    if (b16) v = bf16r(v);
                    y[n] = v;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == ns) { slot = 0; phase ^= 1u; }
    }
    return true;
}



// Eight fp16 weights (one 16-byte piece) against eight activations already
// widened to fp32: the same products and fmaf order as dot8_f16 (an fp16 x
// fp16 product is exact in fp32), with half the conversions.  Callers pass a
// register copy of the piece: a reference bound straight to shared memory
// is read as four 4-byte loads at a 16-byte lane stride (4-way conflicts).
__device__ __forceinline__ float dot8_f16_f32(const int4 &a, const float *x, float acc) {
    const __half2 *ha = reinterpret_cast<const __half2 *>(&a);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 fa = __half22float2(ha[i]);
        acc = fmaf(fa.x, x[2 * i], acc);
        acc = fmaf(fa.y, x[2 * i + 1], acc);
    }
    return acc;
}

// Widens the 16-byte fp16 activation piece p into x[0..8).
__device__ __forceinline__ void widen8_f16(const uint16_t *xh, int p, float *x) {
    const int4 v = *reinterpret_cast<const int4 *>(xh + p * 8);
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(h[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

// Ring position after `chunks` more chunks from (slot, phase): the
// out-of-line ops below take the position by value and the caller advances.
__device__ __forceinline__ void ring_advance(int &slot, uint32_t &phase, int64_t chunks, int ns) {
    const int64_t pos = slot + chunks;
    slot = (int)(pos % ns);
    if ((pos / ns) & 1) phase ^= 1u;
}

// F16 decode fast path (M = 1): as q8_m1_op, LPR lanes own one weight row and
// lane s of a row takes the 16-byte (8-value) pieces s, s+LPR, ...; the
// lane's activation pieces stay in registers, widened to fp32 once per op.
// Each piece contributes eight fp16 x fp16 products accumulated in fp32; a
// row is reduced over its LPR lanes.  EPI_SWIGLU needs RPW even (LPR <= 16).
// Out of line (the 8*IT activation registers); the ring position comes by
// value and the caller advances it by ceil((r1 - r0) / rows_per_chunk).
template <int LPR, int IT>
__device__ __noinline__ bool f16_m1_op(const StreamOp &op, const uint8_t *wslot, const uint16_t *xh,
                                       uint64_t *full, uint64_t *empty, int slot, uint32_t phase, int64_t r0,
                                       int64_t r1, int cw, int lane, volatile int *abort_flag, int *err, int ns) {
    constexpr int RPW = 32 / LPR;
    constexpr int RPP = RPW * ST_CONSUMER_WARPS;
    const int K = op.K;
    const int ls = lane % LPR, lr = lane / LPR;
    float xf[8 * IT];
#pragma unroll
    for (int i = 0; i < IT; i++) widen8_f16(xh, ls + LPR * i, xf + 8 * i);
    float *y = op.y + out_row(op, 0) * op.ldy;
    const float *bias = op.bias;
    const bool b16 = op.flags & VB_OUT_BF16;
    const bool residual = op.epi == EPI_RESIDUAL;
    const bool swz = op.epi == EPI_SWIGLU;
    const int R = op.rows_per_chunk;
    for (int64_t r = r0; r < r1; r += R) {
        const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
        if (!wait_phase(&full[slot], phase, abort_flag)) {
            if (!*abort_flag) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); *abort_flag = 1; }
            return false;
        }
        const uint8_t *wt = wslot + (size_t)slot * ST_SLOT;
        for (int jb = cw * RPW; jb < nr; jb += RPP) {   // warp-uniform
            const int j = jb + lr;
            const bool valid = j < nr;
            const int jj = valid ? j : jb;
            const uint8_t *wr = wt + (int64_t)slot_row(jj, nr, swz) * K * 2;
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < IT; i++) {
                const int4 wv = *reinterpret_cast<const int4 *>(wr + (ls + LPR * i) * 16);   // one 16-byte load
                acc = dot8_f16_f32(wv, xf + 8 * i, acc);
            }
#pragma unroll
            for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (swz) {
                const float up = __shfl_down_sync(0xffffffffu, acc, LPR);   // row j + 1
                if (valid && ls == 0 && !(lr & 1)) swiglu_store(op, 0, (r + j) >> 1, acc, up);
            } else if (valid && ls == 0) {
                const int64_t n = r + j;
                if (residual) {
                    y[n] = stream_epilogue(op, 0, n, acc);
                } else {
                    float v = acc;
                    if (bias) v = __fadd_rn(v, bias[n]);
                    if (b16) v = bf16r(v);
                    y[n] = v;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == ns) { slot = 0; phase ^= 1u; }
    }
    return true;
}

// F16 decode path for long rows (M = 1, K = WPR * 256 * IT): a ring chunk
// holds only R = ST_CONSUMER_WARPS / WPR rows (2 for K 6144/8192, 4 for
// 4096), so WPR warps share a row: warp cw takes row cw / WPR and K segment
// cw % WPR, lane l the 16-byte pieces seg*32*IT + l + 32 i, whose activation
// stays in registers (widened to fp32 once per op).  The segment partials meet in `part` (two buffers of
// ST_CONSUMER_WARPS floats, alternating per chunk) behind one consumer
// barrier per chunk, which also makes a failed wait a uniform exit; the
// segment-0 warp adds them in segment order and stores.  Not for
// EPI_SWIGLU.  Out of line like f16_m1_op (ring position by value, the caller
// advances it).  Returns false on a timeout or an abort.
template <int WPR, int IT>
__device__ __noinline__ bool f16_m1_split_op(const StreamOp &op, const uint8_t *wslot, const uint16_t *xh,
                                             float *part, uint64_t *full, uint64_t *empty, int slot,
                                             uint32_t phase, int64_t r0, int64_t r1, int cw, int lane,
                                             volatile int *abort_flag, int *err, int ns) {
    static_assert(ST_CONSUMER_WARPS % WPR == 0, "warps per row");
    constexpr int R = ST_CONSUMER_WARPS / WPR;   // rows per chunk (checked by the caller)
    constexpr int SEGP = 32 * IT;                 // 16-byte pieces per segment
    const int K = op.K;
    const int seg = cw % WPR, jrow = cw / WPR;
    float xf[8 * IT];
#pragma unroll
    for (int i = 0; i < IT; i++) widen8_f16(xh, seg * SEGP + lane + 32 * i, xf + 8 * i);
    int buf = 0;
    for (int64_t r = r0; r < r1; r += R) {
        const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
        const bool ok = wait_phase(&full[slot], phase, abort_flag);
        if (!ok && !*abort_flag) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); *abort_flag = 1; }
        if (__all_sync(0xffffffffu, ok)) {
            float acc = 0.0f;
            if (jrow < nr) {   // warp-uniform
                const uint8_t *wr = wslot + (size_t)slot * ST_SLOT + (int64_t)jrow * K * 2;
#pragma unroll
                for (int i = 0; i < IT; i++) {
                    const int4 wv = *reinterpret_cast<const int4 *>(wr + (seg * SEGP + lane + 32 * i) * 16);
                    acc = dot8_f16_f32(wv, xf + 8 * i, acc);
                }
                acc = warp_sum(acc);
            }
            __syncwarp();
            if (lane == 0) {
                part[buf * ST_CONSUMER_WARPS + cw] = acc;
                mbar_arrive(&empty[slot]);
            }
        }
        if (consumer_sync_or(!ok, ST_CONSUMERS)) return false;
        if (seg == 0 && jrow < nr && lane == 0) {
            const float *p = part + buf * ST_CONSUMER_WARPS + cw;
            float v = p[0];
#pragma unroll
            for (int s = 1; s < WPR; s++) v += p[s];
            stream_store(op, 0, r + jrow, v);
        }
        buf ^= 1;
        if (++slot == ns) { slot = 0; phase ^= 1u; }
    }
    return true;
}

}  // namespace vb

namespace vb {


__device__ __forceinline__ float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }

// Decode attention geometry (see stream_attn): rows per pass, and the
// spans per (sequence, head) and passes per span for L visible rows.
constexpr int ATT_PASS = 64;

__device__ __forceinline__ void attn_split(int L, int M, int NH, int G, int &nsp, int &ppi) {
    const int passes = (L + ATT_PASS - 1) / ATT_PASS;
    const int cap = max(1, G / (M * NH));
    ppi = (passes + cap - 1) / cap;
    nsp = (passes + ppi - 1) / ppi;
}


// Row scales 1/sqrtf(mean(x^2)+eps) of M rows (the ggml_rms_norm statistic:
// fp32 squares summed in double), left in aux[0..M).  All consumer threads.
__device__ __forceinline__ void stream_row_scales(const float *x, int64_t ldx, int M, int K, float eps, float *aux,
                                                  int ctid, int cw, int lane) {
    double *red = reinterpret_cast<double *>(aux + 16);   // [warps][8]
    for (int m = 0; m < M; m++) {
        double s = 0.0;
        for (int k = ctid; k < K; k += ST_CONSUMERS) {
            const float v = __ldcg(x + (int64_t)m * ldx + k);
            s += (double)__fmul_rn(v, v);
        }
        s = warp_sum_d(s);
        if (lane == 0) red[cw * 8 + m] = s;
    }
    consumer_sync(ST_CONSUMERS);
    if (ctid < M) {
        double t = 0.0;
        for (int w = 0; w < ST_CONSUMER_WARPS; w++) t += red[w * 8 + ctid];
        const float mean = __double2float_rn(__ddiv_rn(t, (double)K));
        aux[ctid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    consumer_sync(ST_CONSUMERS);
}

// Eight consecutive prologue values of row m starting at column k0.
__device__ __forceinline__ void stream_pro_values(const StreamOp &op, int m, int k0, const float *aux, float v[8]) {
    const float *xr = op.x + in_row(op, m) * op.ldx;
    if (op.pro == PRO_SWIGLU) {
        const int F = op.pro_len;
        const float4 g0 = __ldcg(reinterpret_cast<const float4 *>(xr + k0));
        const float4 g1 = __ldcg(reinterpret_cast<const float4 *>(xr + k0 + 4));
        const float4 u0 = __ldcg(reinterpret_cast<const float4 *>(xr + F + k0));
        const float4 u1 = __ldcg(reinterpret_cast<const float4 *>(xr + F + k0 + 4));
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = bf16r(__fmul_rn(bf16r(silu_f(bf16r(g[e]))), bf16r(u[e])));
        return;
    }
    const float4 f0 = __ldcg(reinterpret_cast<const float4 *>(xr + k0));
    const float4 f1 = __ldcg(reinterpret_cast<const float4 *>(xr + k0 + 4));
    const float f[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
    if (op.pro == PRO_RMSNORM) {
        const float sc = aux[m];
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = bf16r(__fmul_rn(bf16r(__fmul_rn(f[e], sc)), __ldg(op.pro_w + k0 + e)));
        return;
    }
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = f[e];
}

// Q8_0 quantization of 8 consecutive values by one of the four threads
// that share a 32-value block (lanes 4k..4k+3): ggml's rule, bit-exact.
// All 32 lanes must call it (the block maximum is a shuffle reduction).
__device__ __forceinline__ void q8_store8(const float v[8], bool valid, int qrule, int8_t *dst, float *dscale,
                                          bool first) {
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(v[e]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const uint16_t dh = f2h(d);
    const bool x86 = qrule == VB_QRULE_X86;
    float id;
    if (x86) id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t pk[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t w4 = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float t = __fmul_rn(v[4 * h + e], id);
            const int q = x86 ? __float2int_rn(t) : (int)roundf(t);
            w4 |= ((uint32_t)(q & 0xff)) << (8 * e);
        }
        pk[h] = w4;
    }
    if (valid) {
        *reinterpret_cast<uint2 *>(dst) = make_uint2(pk[0], pk[1]);
        if (first) *dscale = h2f(dh);
    }
}


// R rounds (items r0*256 + ctid, (r0+1)*256 + ctid, ...) of the Q8_0
// prologue with every global load issued before any arithmetic, so a round
// costs one memory latency in total rather than one each.  Item = 8 values
// (a quarter of a 32-value block) of row m.  With fused_norm the RMSNorm row
// statistics are computed here from the loaded values (requires all items
// in this batch and K % 256 == 0, so a warp's 32 items share one row);
// otherwise aux[m] already holds them.
template <int R>
__device__ __forceinline__ void q8_prologue_batch(const StreamOp &op, int r0, bool fused_norm, int8_t *xq, float *xd,
                                                  float *aux, int ctid, int cw, int lane) {
    const int K = op.K, M = op.M, nb = K >> 5, ipr = nb * 4, total = M * ipr, pro = op.pro;
    float4 a[R][2], b[R][2];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int it = (r0 + r) * ST_CONSUMERS + ctid;
        a[r][0] = a[r][1] = b[r][0] = b[r][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (it < total) {
            const int m = it / ipr, k0 = (it - m * ipr) * 8;
            const float *xr = op.x + in_row(op, m) * op.ldx + k0;
            a[r][0] = ldcg4(xr);
            a[r][1] = ldcg4(xr + 4);
            if (pro == PRO_SWIGLU) {
                b[r][0] = ldcg4(xr + op.pro_len);
                b[r][1] = ldcg4(xr + op.pro_len + 4);
            } else if (pro == PRO_RMSNORM) {
                b[r][0] = __ldg(reinterpret_cast<const float4 *>(op.pro_w + k0));
                b[r][1] = __ldg(reinterpret_cast<const float4 *>(op.pro_w + k0 + 4));
            }
        }
    }
    if (fused_norm) {
        // fp32 squares summed in double: per warp-round, then per row in a
        // fixed order (deterministic)
        double *red = reinterpret_cast<double *>(aux + 16);   // [R][warps]
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float f[8] = {a[r][0].x, a[r][0].y, a[r][0].z, a[r][0].w, a[r][1].x, a[r][1].y, a[r][1].z, a[r][1].w};
            double sq = 0.0;
#pragma unroll
            for (int e = 0; e < 8; e++) sq += (double)__fmul_rn(f[e], f[e]);
            sq = warp_sum_d(sq);
            if (lane == 0) red[r * ST_CONSUMER_WARPS + cw] = sq;
        }
        consumer_sync(ST_CONSUMERS);
        if (cw == 0) {
            // warp 0: lane j holds warp-round j's partial (R * 8 <= 32);
            // each row's total is a fixed-order tree sum, then lane m
            // finishes row m.  Division by K is a multiplication when K is
            // a power of two (exact).
            const int it0 = (r0 + lane / ST_CONSUMER_WARPS) * ST_CONSUMERS + (lane % ST_CONSUMER_WARPS) * 32;
            const bool have = lane < R * ST_CONSUMER_WARPS && it0 < total;
            const double part = have ? red[lane] : 0.0;
            const int row = have ? it0 / ipr : -1;
            double mine = 0.0;
            for (int mm = 0; mm < M; mm++) {
                const double t = warp_sum_d(row == mm ? part : 0.0);
                if (lane == mm) mine = t;
            }
            if (lane < M) {
                const double md = (K & (K - 1)) == 0 ? __dmul_rn(mine, 1.0 / (double)K) : __ddiv_rn(mine, (double)K);
                aux[lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(md), op.eps)));
            }
        }
        consumer_sync(ST_CONSUMERS);
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int it = (r0 + r) * ST_CONSUMERS + ctid;
        const bool valid = it < total;
        const int itc = valid ? it : 0;
        const int m = itc / ipr, q = itc - m * ipr, kb = q >> 2, part = q & 3;
        const float f[8] = {a[r][0].x, a[r][0].y, a[r][0].z, a[r][0].w, a[r][1].x, a[r][1].y, a[r][1].z, a[r][1].w};
        const float g[8] = {b[r][0].x, b[r][0].y, b[r][0].z, b[r][0].w, b[r][1].x, b[r][1].y, b[r][1].z, b[r][1].w};
        float v[8];
        if (pro == PRO_SWIGLU) {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = bf16r(__fmul_rn(bf16r(silu_f(bf16r(f[e]))), bf16r(g[e])));
        } else if (pro == PRO_RMSNORM) {
            const float sc = aux[m];
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = bf16r(__fmul_rn(bf16r(__fmul_rn(f[e], sc)), g[e]));
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = f[e];
        }
        q8_store8(v, valid, op.qrule, xq + (int64_t)m * K + kb * QK + part * 8, xd + m * nb + kb, part == 0);
    }
}

// The activation operand of a GEMV op for all M rows: prologue values,
// then ggml's Q8_0 rule (four threads per 32-value block, bit-exact) or the
// fp16 rounding of an F16 op.  Requires K % 32 == 0 except for a plain
// F16 load.  Ends with a consumer barrier.
__device__ __noinline__ void stream_prologue(const StreamOp &op, int8_t *xq, float *xd, float *aux, int ctid, int cw,
                                             int lane) {
    const int K = op.K, M = op.M, nb = K / QK;
    if (op.wtype == VB_TYPE_Q8_0) {
        const int rounds = (M * nb * 4 + ST_CONSUMERS - 1) / ST_CONSUMERS;
        const bool fused = op.pro == PRO_RMSNORM && rounds <= 4 && (K % 256) == 0;
        if (op.pro == PRO_RMSNORM && !fused) stream_row_scales(op.x, op.ldx, M, K, op.eps, aux, ctid, cw, lane);
        for (int r0 = 0; r0 < rounds; r0 += 4) {
            switch (min(4, rounds - r0)) {
                case 1: q8_prologue_batch<1>(op, r0, fused, xq, xd, aux, ctid, cw, lane); break;
                case 2: q8_prologue_batch<2>(op, r0, fused, xq, xd, aux, ctid, cw, lane); break;
                case 3: q8_prologue_batch<3>(op, r0, fused, xq, xd, aux, ctid, cw, lane); break;
                default: q8_prologue_batch<4>(op, r0, fused, xq, xd, aux, ctid, cw, lane); break;
            }
        }
        consumer_sync(ST_CONSUMERS);
        return;
    }
    // F16 operand: fp16 values of the prologue output
    if (op.pro == PRO_RMSNORM) stream_row_scales(op.x, op.ldx, M, K, op.eps, aux, ctid, cw, lane);
    uint16_t *xh = reinterpret_cast<uint16_t *>(xq);
    for (int e = ctid; e < M * K / 8; e += ST_CONSUMERS) {
        const int m = (e * 8) / K, k = (e * 8) % K;
        float v[8];
        stream_pro_values(op, m, k, aux, v);
        uint4 o;
        o.x = (uint32_t)f2h(v[0]) | ((uint32_t)f2h(v[1]) << 16);
        o.y = (uint32_t)f2h(v[2]) | ((uint32_t)f2h(v[3]) << 16);
        o.z = (uint32_t)f2h(v[4]) | ((uint32_t)f2h(v[5]) << 16);
        o.w = (uint32_t)f2h(v[6]) | ((uint32_t)f2h(v[7]) << 16);
        *reinterpret_cast<uint4 *>(xh + (int64_t)m * K + k) = o;
    }
    consumer_sync(ST_CONSUMERS);
}

// NEOX rotation of one pair with the host-built table, bf16-rounded
// (src/minicpm4.c:205-222).
__device__ __forceinline__ void rope_pair(float x0, float x1, const float *cs, int p, float &r0, float &r1) {
    const float c = cs[2 * p], s = cs[2 * p + 1];
    r0 = bf16r(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
    r1 = bf16r(__fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
}

// Decode attention inside the persistent kernel (vcpm_attention for one new
// token per sequence, src/minicpm4.c:250-428): for query head h of KV group
// g = h / (n_heads / n_kv), s_l = (q . k_l) / sqrt(head_dim) and
// o = softmax(s) . V over the sequence's visible rows.
//
// Work items are (sequence, head, row span); the spans are as long as it
// takes for every item to fit in one wave of the grid (attn_split), so no
// CTA runs two items.  An item walks its span in passes of ATT_PASS rows
// with an online softmax (running max and sum, the partial output rescaled
// when the max grows).  A pass loads its K and V words straight into
// registers -- K as four threads per row (a quarter of the dimensions
// each), V as four consecutive words per thread over a subset of the rows
// -- all issued before any arithmetic, so a pass costs one memory latency.
// The new token's row comes from this step's k/v (rotated, bf16), and the
// group's first head appends it to the cache.  A head with one span writes
// its output directly; otherwise each item writes its (max, sum) and
// partial output, and the item that finishes a (sequence, head) last (a
// device-wide count, no waiting) merges the spans into y.  op.eps carries
// the score scale 1/sqrt(head_dim); st holds the step's [M][4] row
// parameters (shared memory).  head_dim is 64, 128 or 256.
template <int HW>
__device__ __forceinline__ void stream_attn_hw(const StreamOp &op, const int *st, uint8_t *aux, int cta, int G,
                                               int ctid, int cw, int lane) {
    __shared__ int s_last;
    __shared__ float s_l;
    constexpr int HD = 2 * HW, HALF = HW;
    constexpr int KW = HW / 4;                  // K words per thread (four threads per row)
    constexpr int VG = HW / 4;                  // V word groups of 4
    constexpr int VR = ST_CONSUMERS / VG;       // V row subsets
    constexpr int VJ = ATT_PASS / VR;           // V rows per thread
    static_assert(ST_CONSUMERS == 4 * ATT_PASS, "one K quarter-row per thread");
    const int NH = op.n_heads, qpk = NH / op.n_kv;
    const int QD = NH * HD, KD = op.n_kv * HD;
    float *qs = reinterpret_cast<float *>(aux);                     // [HD] rotated query
    uint32_t *fk = reinterpret_cast<uint32_t *>(qs + HD);          // [HW] new row, K words
    uint32_t *fv = fk + HW;                                         // [HW] new row, V words
    float *scs = reinterpret_cast<float *>(fv + HW);                // [ATT_PASS] scores
    float2 *vred = reinterpret_cast<float2 *>(scs + ATT_PASS);     // [warps][HW] partial outputs
    const uint32_t *kc32 = reinterpret_cast<const uint32_t *>(op.kc);
    const uint32_t *vc32 = reinterpret_cast<const uint32_t *>(op.vc);
    // thread roles: K row kr, quarter kq; V word group vg, row subset vq
    const int kr = ctid >> 2, kq = ctid & 3;
    const int vg = ctid % VG, vq = ctid / VG;
    int base = 0;   // first item index of sequence m
    for (int m = 0; m < op.M; m++) {
        const int rope_pos = st[4 * m], wrow = st[4 * m + 1], rstart = st[4 * m + 2], L = st[4 * m + 3];
        int nsp, ppi;
        attn_split(L, op.M, NH, G, nsp, ppi);
        const float *qrow = op.qkv + (int64_t)m * op.ldqkv;
        const float *cs = op.rope_cs + (int64_t)rope_pos * HD;
        const int fresh = wrow - rstart;
        const int items = NH * nsp;
        for (int idx = base + (cta - base % G + G) % G; idx < base + items; idx += G) {
            const int h = (idx - base) / nsp, sp = (idx - base) - h * nsp, g = h / qpk;
            const int row0 = sp * ppi * ATT_PASS, row1 = min(L, row0 + ppi * ATT_PASS);
            const uint32_t *kg32 = kc32 + ((int64_t)g * op.n_rows + rstart) * HW;
            const uint32_t *vg32 = vc32 + ((int64_t)g * op.n_rows + rstart) * HW;
            consumer_sync(ST_CONSUMERS);   // the previous item's readers of qs / fk / vred are done
            float mrun = -INFINITY, lrun = 0.0f;
            float ox[4] = {0.f, 0.f, 0.f, 0.f}, oy[4] = {0.f, 0.f, 0.f, 0.f};
            for (int p0 = row0; p0 < row1; p0 += ATT_PASS) {
                const int n = min(ATT_PASS, row1 - p0);
                // ---- loads of the pass (cache rows; the new row is patched below)
                uint4 kw[KW / 4];
                uint4 vw[VJ];
#pragma unroll
                for (int t = 0; t < KW / 4; t++) {
                    kw[t] = make_uint4(0u, 0u, 0u, 0u);
                    if (kr < n)
                        kw[t] = __ldcg(reinterpret_cast<const uint4 *>(kg32 + (int64_t)(p0 + kr) * HW + kq * KW) + t);
                }
#pragma unroll
                for (int j = 0; j < VJ; j++) {
                    const int r = vq + j * VR;
                    vw[j] = make_uint4(0u, 0u, 0u, 0u);
                    if (r < n) vw[j] = __ldcg(reinterpret_cast<const uint4 *>(vg32 + (int64_t)(p0 + r) * HW) + vg);
                }
                if (p0 == row0) {
                    // rotated query, and the new row if it is in this span
                    for (int p = ctid; p < HALF; p += ST_CONSUMERS) {
                        const float x0 = __ldcg(qrow + h * HD + p), x1 = __ldcg(qrow + h * HD + p + HALF);
                        float r0 = x0, r1 = x1;
                        if (op.use_rope) rope_pair(x0, x1, cs, p, r0, r1);
                        qs[p] = r0;
                        qs[p + HALF] = r1;
                    }
                    if (fresh >= row0 && fresh < row1) {
                        uint16_t *k16 = reinterpret_cast<uint16_t *>(fk);
                        uint16_t *v16 = reinterpret_cast<uint16_t *>(fv);
                        const bool owner = (h % qpk) == 0;   // appends the row to the cache
                        uint16_t *kgw = op.kc + ((int64_t)g * op.n_rows + wrow) * HD;
                        uint16_t *vgw = op.vc + ((int64_t)g * op.n_rows + wrow) * HD;
                        for (int p = ctid; p < HALF; p += ST_CONSUMERS) {
                            const float k0 = __ldcg(qrow + QD + g * HD + p), k1 = __ldcg(qrow + QD + g * HD + p + HALF);
                            float r0 = bf16r(k0), r1 = bf16r(k1);
                            if (op.use_rope) rope_pair(k0, k1, cs, p, r0, r1);
                            const uint16_t b0 = bf16_bits(r0), b1 = bf16_bits(r1);
                            const uint16_t c0 = bf16_bits(__ldcg(qrow + QD + KD + g * HD + p));
                            const uint16_t c1 = bf16_bits(__ldcg(qrow + QD + KD + g * HD + p + HALF));
                            k16[p] = b0;
                            k16[p + HALF] = b1;
                            v16[p] = c0;
                            v16[p + HALF] = c1;
                            if (owner) {
                                kgw[p] = b0;
                                kgw[p + HALF] = b1;
                                vgw[p] = c0;
                                vgw[p + HALF] = c1;
                            }
                        }
                    }
                    consumer_sync(ST_CONSUMERS);
                }
                if (fresh >= p0 && fresh < p0 + n) {
                    if (kr == fresh - p0) {
#pragma unroll
                        for (int t = 0; t < KW / 4; t++)
                            kw[t] = reinterpret_cast<const uint4 *>(fk + kq * KW)[t];
                    }
#pragma unroll
                    for (int j = 0; j < VJ; j++)
                        if (vq + j * VR == fresh - p0) vw[j] = reinterpret_cast<const uint4 *>(fv)[vg];
                }
                // ---- scores: four threads per row, two shuffles
                {
                    const float2 *qv = reinterpret_cast<const float2 *>(qs) + kq * KW;
                    float a = 0.0f;
#pragma unroll
                    for (int t = 0; t < KW / 4; t++) {
                        const uint32_t wds[4] = {kw[t].x, kw[t].y, kw[t].z, kw[t].w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float2 q = qv[4 * t + e];
                            a = fmaf(__uint_as_float(wds[e] << 16), q.x, a);
                            a = fmaf(__uint_as_float(wds[e] & 0xffff0000u), q.y, a);
                        }
                    }
                    a += __shfl_xor_sync(0xffffffffu, a, 1);
                    a += __shfl_xor_sync(0xffffffffu, a, 2);
                    if (kq == 0) scs[kr] = (kr < n) ? __fmul_rn(a, op.eps) : -INFINITY;
                }
                consumer_sync(ST_CONSUMERS);
                // ---- online softmax, identical in every warp (rows lane, lane + 32)
                const float s0 = scs[lane], s1 = scs[lane + 32];
                const float pmax = warp_max(fmaxf(s0, s1));
                const float mnew = fmaxf(mrun, pmax);
                const float fac = mrun == -INFINITY ? 0.0f : expf(mrun - mnew);
                const float e0 = lane < n ? expf(s0 - mnew) : 0.0f;
                const float e1 = lane + 32 < n ? expf(s1 - mnew) : 0.0f;
                lrun = fmaf(lrun, fac, warp_sum(e0 + e1));
                mrun = mnew;
                // ---- values: rows vq + j * VR, words 4 vg .. 4 vg + 3
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    ox[e] *= fac;
                    oy[e] *= fac;
                }
#pragma unroll
                for (int j = 0; j < VJ; j++) {
                    const int r = vq + j * VR;
                    const float ea = __shfl_sync(0xffffffffu, e0, r & 31);
                    const float eb = __shfl_sync(0xffffffffu, e1, r & 31);
                    const float ep = r < 32 ? ea : eb;
                    const uint32_t wds[4] = {vw[j].x, vw[j].y, vw[j].z, vw[j].w};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        ox[e] = fmaf(ep, __uint_as_float(wds[e] << 16), ox[e]);
                        oy[e] = fmaf(ep, __uint_as_float(wds[e] & 0xffff0000u), oy[e]);
                    }
                }
                consumer_sync(ST_CONSUMERS);   // scs is rewritten by the next pass
            }
            // ---- partial output of the span: sum the row subsets
#pragma unroll
            for (int sh = VG; sh < 32; sh <<= 1) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    ox[e] += __shfl_xor_sync(0xffffffffu, ox[e], sh);
                    oy[e] += __shfl_xor_sync(0xffffffffu, oy[e], sh);
                }
            }
            if (lane < VG) {
#pragma unroll
                for (int e = 0; e < 4; e++) vred[cw * HW + 4 * vg + e] = make_float2(ox[e], oy[e]);
            }
            consumer_sync(ST_CONSUMERS);
            float2 o = make_float2(0.f, 0.f);
            if (ctid < HW) {
                o = vred[ctid];
                for (int w2 = 1; w2 < ST_CONSUMER_WARPS; w2++) {
                    const float2 t = vred[w2 * HW + ctid];
                    o.x = __fadd_rn(o.x, t.x);
                    o.y = __fadd_rn(o.y, t.y);
                }
            }
            if (nsp == 1) {
                // one span: the item's output is the head's
                if (ctid < HW)
                    *reinterpret_cast<float2 *>(op.y + (int64_t)m * op.ldy + h * HD + 2 * ctid) =
                        make_float2(__fdiv_rn(o.x, lrun), __fdiv_rn(o.y, lrun));
                continue;
            }
            const int64_t pi = ((int64_t)m * NH + h) * op.max_chunks + sp;
            if (ctid < HW) *reinterpret_cast<float2 *>(op.part + pi * HD + 2 * ctid) = o;
            if (ctid == 0) *reinterpret_cast<float2 *>(op.part_ml + pi * 2) = make_float2(mrun, lrun);
            // Count the item once the CTA's partials are released (barrier,
            // then a cumulative fence); the last item of the (sequence,
            // head) acquires everyone's and merges the spans.
            consumer_sync(ST_CONSUMERS);
            if (ctid == 0) {
                fence_acq_rel_gpu();
                s_last = atomicAdd(op.cnt + m * NH + h, 1u) == (unsigned)(nsp - 1);
                if (s_last) fence_acq_rel_gpu();
            }
            consumer_sync(ST_CONSUMERS);
            if (s_last) {
                // thread (d4, sl): 4 dims of spans sl, sl + S, ...
                const int D4 = HD >> 2, S = ST_CONSUMERS / D4, d4 = ctid % D4, sl = ctid / D4;
                const float *po = op.part + ((int64_t)m * NH + h) * op.max_chunks * HD + 4 * d4;
                const float *pml = op.part_ml + ((int64_t)m * NH + h) * op.max_chunks * 2;
                const int mc4 = (op.max_chunks + 3) & ~3;
                float *cm = reinterpret_cast<float *>(aux);            // [max_chunks] max -> factor
                float *cl = cm + mc4;                                   // [max_chunks] sum
                float4 *sred = reinterpret_cast<float4 *>(cl + mc4);   // [S][D4]
                for (int t = ctid; t < nsp; t += ST_CONSUMERS) {
                    const float2 ml = __ldcg(reinterpret_cast<const float2 *>(pml) + t);
                    cm[t] = ml.x;
                    cl[t] = ml.y;
                }
                consumer_sync(ST_CONSUMERS);
                if (cw == 0) {
                    float gm = -INFINITY;
                    for (int c2 = lane; c2 < nsp; c2 += 32) gm = fmaxf(gm, cm[c2]);
                    gm = warp_max(gm);
                    float gl = 0.0f;
                    for (int c2 = lane; c2 < nsp; c2 += 32) {
                        const float f = expf(cm[c2] - gm);
                        gl = fmaf(cl[c2], f, gl);
                        cm[c2] = f;
                    }
                    gl = warp_sum(gl);
                    if (lane == 0) s_l = gl;
                }
                consumer_sync(ST_CONSUMERS);
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int c2 = sl; c2 < nsp; c2 += S) {
                    const float4 ov = ldcg4(po + (int64_t)c2 * HD);
                    const float f = cm[c2];
                    acc.x = fmaf(ov.x, f, acc.x);
                    acc.y = fmaf(ov.y, f, acc.y);
                    acc.z = fmaf(ov.z, f, acc.z);
                    acc.w = fmaf(ov.w, f, acc.w);
                }
                sred[sl * D4 + d4] = acc;
                consumer_sync(ST_CONSUMERS);
                if (ctid < HD) {
                    const float *sr = reinterpret_cast<const float *>(sred);
                    float o2 = 0.0f;
                    for (int s2 = 0; s2 < S; s2++) o2 = __fadd_rn(o2, sr[s2 * HD + ctid]);
                    op.y[(int64_t)m * op.ldy + h * HD + ctid] = __fdiv_rn(o2, s_l);
                }
            }
        }
        base += items;
    }
}

__device__ __noinline__ void stream_attn(const StreamOp &op, const int *st, uint8_t *aux, int cta, int G, int ctid,
                                         int cw, int lane) {
    switch (op.head_dim) {
        case 64: stream_attn_hw<32>(op, st, aux, cta, G, ctid, cw, lane); break;
        case 128: stream_attn_hw<64>(op, st, aux, cta, G, ctid, cw, lane); break;
        default: stream_attn_hw<128>(op, st, aux, cta, G, ctid, cw, lane); break;
    }
}

// L2 prefetch of the K/V rows (and RoPE row) this CTA's attention items
// will read: issued by the producer thread when it passes the op, a few
// microseconds before the consumers get there.  Same item enumeration as
// stream_attn.  Requires head_dim % 8 == 0 (16-byte rows).
__device__ __forceinline__ void attn_prefetch(const StreamOp &op, const int *st, int cta, int G) {
    const int HD = op.head_dim, NH = op.n_heads, qpk = NH / op.n_kv;
    int base = 0;
    for (int m = 0; m < op.M; m++) {
        const int rope_pos = st[4 * m], rstart = st[4 * m + 2], L = st[4 * m + 3];
        int nsp, ppi;
        attn_split(L, op.M, NH, G, nsp, ppi);
        const int items = NH * nsp;
        for (int idx = base + (cta - base % G + G) % G; idx < base + items; idx += G) {
            const int h = (idx - base) / nsp, sp = (idx - base) - h * nsp;
            const int row0 = sp * ppi * ATT_PASS, n = min(L, row0 + ppi * ATT_PASS) - row0;
            const int64_t row = (int64_t)(h / qpk) * op.n_rows + rstart + row0;
            prefetch_l2(op.kc + row * HD, (uint32_t)(n * HD * 2));
            prefetch_l2(op.vc + row * HD, (uint32_t)(n * HD * 2));
            if (op.use_rope) prefetch_l2(op.rope_cs + (int64_t)rope_pos * HD, (uint32_t)(HD * 4));
        }
        base += items;
    }
}

// y = bf16(bf16(rms_norm(x)) * w) for rows m = cta, cta + G, ... (final norm).
__device__ __noinline__ void stream_norm(const StreamOp &op, float *aux, int cta, int G, int ctid, int cw, int lane) {
    for (int m = cta; m < op.M; m += G) {   // CTA-uniform
        stream_row_scales(op.x + (int64_t)m * op.ldx, op.ldx, 1, op.K, op.eps, aux, ctid, cw, lane);
        const float sc = aux[0];
        for (int k = ctid; k < op.K; k += ST_CONSUMERS) {
            const float v = __ldcg(op.x + (int64_t)m * op.ldx + k);
            op.y[(int64_t)m * op.ldy + k] = bf16r(__fmul_rn(bf16r(__fmul_rn(v, sc)), __ldg(op.pro_w + k)));
        }
        consumer_sync(ST_CONSUMERS);
    }
}

}  // namespace vb
