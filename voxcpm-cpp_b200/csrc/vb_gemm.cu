// vb_gemm.cu -- tensor-core mat-mul (tcgen05 + TMEM + TMA) for M >= 16
// activation rows: prefill, CFG-batched LocDiT evaluations, multi-request
// decode batches.  The M < 16 decode shapes stay on the weight-streaming
// GEMV kernels.
//
// ggml semantics (src/minicpm4.c:270-458, src/locdit.c:150-391 call sites):
//   Q8_0 weight: y[m][n] = sum_b d_w[n,b] * d_x[m,b] * sum_{j<32} qw[n,b,j] * qx[m,b,j]
//                where (qx, d_x) is the Q8_0 quantization of x (ctx rule);
//   F16 weight:  y[m][n] = sum_k w[n][k] * fp16(x[m][k]), fp32 accumulation.
//
// F16 runs as kind::f16 MMAs on the weights and fp16(x) directly: every
// product is exact in fp32, as in the reference.
//
// Q8_0: the per-block scale pairs rule out accumulating integer products
// across blocks, so both operands are dequantised per block to their exact
// fp32 values v = d * q (an int8 times an fp16 needs 18 significant bits)
// and each v is split into two fp16 terms v = hi + lo (hi = fp16(v),
// lo = fp16(v - hi), exact up to fp16 subnormal spacing).  Three kind::f16
// MMAs per k-step, hi*hi + hi*lo + lo*hi, give every product to about 2^-22
// relative, accumulated in fp32 in TMEM: the result matches ggml's block
// dot up to the fp32 accumulation order.  The activation side is prepared
// once per call (gemm_act_kernel); weight tiles are converted in shared
// memory as they stream in, so HBM carries Q8_0 bytes only.
//
// Tile: 128 weight rows (MMA M = TMEM lanes) x BN activation rows (MMA N =
// TMEM columns, 16..256) x 64 k per stage (one 128-byte swizzle row of
// fp16).  Warp 0 issues TMA loads, warp 1 allocates TMEM and issues MMAs
// (one thread), warps 2..9 convert weight tiles and run the epilogue.  When
// the tile grid is small the K range is split over CTAs; partial sums go to
// a workspace and the last CTA of a tile (device-wide count) adds them in
// split order, so results are deterministic.
#include <cuda.h>

#include <mutex>

#include "vb_common.cuh"
#include "vb_device.cuh"
#include "vb_kernels.cuh"
#include "vb_stream.cuh"

namespace vb {

constexpr int GM_BM = 128;
constexpr int GM_BK = 64;
constexpr int GM_THREADS = 448;        // warp 0 TMA, 1 MMA + TMEM, 2..9 convert, 10..13 epilogue
constexpr int GM_CONV_THREADS = 256;
constexpr int GM_EPI_THREADS = 128;
constexpr int GM_MAX_STAGES = 6;
constexpr int GM_SMEM_BUDGET = 220 * 1024;

struct GemmArgs {
    int q8;                 // 1: Q8_0 weights (hi/lo split), 0: F16 weights
    int bk;                 // k elements per stage (64 fp16 / 32 tf32: one 128-byte swizzle row)
    int K, N, M, BN;
    int kt_total, kt_per_split, splits, tiles_m, tiles_n;
    int n_tma, n_conv;      // pipeline depths
    uint32_t tmem_cols;
    const uint16_t *sc;     // Q8_0 scales [N][K/32]
    float *y;
    const float *bias;
    unsigned flags;
    const float *res;       // residual epilogue source (rows like y) or null
    float res_scale;
    int64_t ldy, seg, seg_stride, seg_off;
    int seg_plain;          // output row = activation row
    float *ws;              // split partials [splits][N][Mp]
    int Mp;                 // tiles_m * BN
    unsigned *cnt;          // per-tile arrival counters (self-resetting)
    int *err;
    // AudioVAE epilogue (the tf32 instantiation): v = acc + bias[n % cb]
    // (+ skip); y = v (if y); out_x = snake(alpha)(sr(v)) (if out_x)
    int cb;
    uint32_t small_off;     // Q8_0 / tf32: TMEM column offset of the cross-term accumulator (hi*lo + lo*hi)
    const float *skip;
    float *out_x;
    const float *alpha, *sr_scale, *sr_bias;
};

__device__ __forceinline__ uint64_t sw128_desc(const void *p) {
    uint64_t d = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                 // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Programmatic dependent launch: kernels of the M >= 16 chain are launched
// so that they may start while the previous kernel of the stream finishes;
// this waits until that kernel has completed and its writes are visible
// (a no-op when the launch was not programmatic).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next programmatic launch of the stream begin scheduling its CTAs
// (they still wait for this grid to complete before touching memory).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The load and its wait are one asm statement: the destination registers
// are written asynchronously until tcgen05.wait::ld, and with two
// statements the compiler may schedule a use of a register between them.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// Bounded mbarrier wait (no abort flag: every role of the CTA reaches the
// teardown on its own once its waits have ended).
__device__ __forceinline__ bool gm_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
    return true;
}

__device__ __forceinline__ int64_t gm_out_row(const GemmArgs &a, int m) {
    if (a.seg_plain) return m;
    const int sg = (int)a.seg;
    return (int64_t)(m / sg) * a.seg_stride + a.seg_off + (m % sg);
}

// Epilogue of 16 outputs (activation rows m0 .. m0+15, weight row n).  The
// residual rows are all loaded before any store: they may alias y, so
// interleaving would serialise 16 memory round trips.
__device__ __forceinline__ void gm_store16(const GemmArgs &a, int m0, int n, const float *acc) {
    float r[16];
    if (a.res) {
#pragma unroll
        for (int cc = 0; cc < 16; cc++) r[cc] = __ldcg(a.res + gm_out_row(a, min(m0 + cc, a.M - 1)) * a.ldy + n);
    }
    const float b = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
    for (int cc = 0; cc < 16; cc++) {
        if (m0 + cc >= a.M) break;
        float v = acc[cc];
        if (a.bias) v = __fadd_rn(v, b);
        if (a.flags & VB_OUT_BF16) v = bf16r(v);
        if (a.res) {
            if (a.res_scale != 1.0f) v = __fmul_rn(v, a.res_scale);
            v = bf16r(__fadd_rn(r[cc], v));
        }
        a.y[gm_out_row(a, m0 + cc) * a.ldy + n] = v;
    }
}

// The same epilogue for 8 outputs (activation rows m0 .. m0+7).
__device__ __forceinline__ void gm_store8(const GemmArgs &a, int m0, int n, const float *acc) {
    float r[8];
    if (a.res) {
#pragma unroll
        for (int cc = 0; cc < 8; cc++) r[cc] = __ldcg(a.res + gm_out_row(a, min(m0 + cc, a.M - 1)) * a.ldy + n);
    }
    const float b = a.bias ? a.bias[n] : 0.0f;
#pragma unroll
    for (int cc = 0; cc < 8; cc++) {
        if (m0 + cc >= a.M) break;
        float v = acc[cc];
        if (a.bias) v = __fadd_rn(v, b);
        if (a.flags & VB_OUT_BF16) v = bf16r(v);
        if (a.res) {
            if (a.res_scale != 1.0f) v = __fmul_rn(v, a.res_scale);
            v = bf16r(__fadd_rn(r[cc], v));
        }
        a.y[gm_out_row(a, m0 + cc) * a.ldy + n] = v;
    }
}

// snake(x, a) = x + sin(a*x)^2 / a, one fp32 op at a time (the AudioVAE
// activation, src/audio_vae_v2.c:483-503).
__device__ __forceinline__ float gm_snake(float x, float al) {
    const float t = __fmul_rn(x, al);
    const float st = sinf(t);
    return __fadd_rn(x, __fdiv_rn(__fmul_rn(st, st), al));
}

// AudioVAE epilogue of 16 outputs (activation rows m0 .. m0+15, output
// channel n): bias, residual skip, the value, and the next layer's input.
// Every skip row is loaded before any store (the skip may alias y).
__device__ __forceinline__ void gm_store16_vae(const GemmArgs &a, int m0, int n, const float *acc) {
    const int c = n % a.cb;
    float r[16];
    if (a.skip) {
#pragma unroll
        for (int cc = 0; cc < 16; cc++) r[cc] = __ldcg(a.skip + (int64_t)min(m0 + cc, a.M - 1) * a.ldy + n);
    }
    const float b = a.bias ? a.bias[c] : 0.0f;
    const float al = a.alpha ? a.alpha[c] : 1.0f;
    const float ss = a.sr_scale ? a.sr_scale[c] : 1.0f, sb = a.sr_scale ? a.sr_bias[c] : 0.0f;
#pragma unroll
    for (int cc = 0; cc < 16; cc++) {
        if (m0 + cc >= a.M) break;
        float v = acc[cc];
        if (a.bias) v = __fadd_rn(v, b);
        if (a.skip) v = __fadd_rn(r[cc], v);
        const int64_t at = (int64_t)(m0 + cc) * a.ldy + n;
        if (a.y) a.y[at] = v;
        if (a.out_x) {
            float u = v;
            if (a.sr_scale) u = __fadd_rn(__fmul_rn(u, ss), sb);
            if (a.alpha) u = gm_snake(u, al);
            a.out_x[at] = u;
        }
    }
}

template <bool TF32>
__device__ __forceinline__ void gm_store(const GemmArgs &a, int m0, int n, const float *acc) {
    if constexpr (TF32) gm_store16_vae(a, m0, n, acc);
    else gm_store16(a, m0, n, acc);
}

// TF32 = false: F16 / Q8_0 weights (a.q8) with the ggml epilogue;
// TF32 = true: tf32 hi/lo operands with the AudioVAE epilogue.  Two
// instantiations, so neither pays the other's registers.
template <bool TF32>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wl,
                const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_bl,
                const GemmArgs a) {
    extern __shared__ uint8_t gsm_raw[];
    uint8_t *gsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bars[4 * GM_MAX_STAGES + 4];
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;
    uint64_t *full = bars, *empty = bars + GM_MAX_STAGES, *cfull = bars + 2 * GM_MAX_STAGES,
             *cempty = bars + 3 * GM_MAX_STAGES, *tfull = bars + 4 * GM_MAX_STAGES, *tempty = tfull + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int BN = a.BN;
    // stage: weight tile (raw int8, fp16, or tf32 hi then lo), activation
    // tile(s) (hi, then lo for Q8_0 / tf32); every row one 128-byte
    // swizzle row
    const uint32_t a_bytes = a.q8 ? GM_BM * GM_BK : GM_BM * 128;
    const uint32_t a_parts = TF32 ? 2u : 1u;
    const uint32_t b_bytes = (uint32_t)BN * 128;
    const uint32_t stage_bytes = a_bytes * a_parts + b_bytes * ((a.q8 || TF32) ? 2 : 1);
    uint8_t *conv = gsm + (size_t)a.n_tma * stage_bytes;                 // converted A: [n_conv][hi 16K | lo 16K]
    const int n_tiles = a.tiles_n * a.tiles_m * a.splits;
    const uint32_t acc_cols = a.tmem_cols >> 1;                         // two accumulators

    if (threadIdx.x == 0) {
        for (int s = 0; s < GM_MAX_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&cfull[s], GM_CONV_THREADS / 32);
            mbar_init(&cempty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], GM_EPI_THREADS / 32);
        }
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    // everything above (barrier init, TMEM allocation) overlaps the previous
    // kernel; operands and outputs are touched only after it has finished
    pdl_wait();
    pdl_trigger();

    // Tiles t = blockIdx.x, + gridDim.x, ...; split fastest, then the
    // activation tile, so CTAs running at the same time share weight tiles.
    auto coords = [&](int t, int &n0, int &m0, int &split, int &kt0, int &nkt) {
        split = t % a.splits;
        t /= a.splits;
        m0 = (t % a.tiles_m) * BN;
        n0 = (t / a.tiles_m) * GM_BM;
        kt0 = split * a.kt_per_split;
        nkt = min(a.kt_per_split, a.kt_total - kt0);
    };

    if (warp == 0) {
        // ---------------------------------------------------------- TMA
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                int n0, m0, split, kt0, nkt;
                coords(t, n0, m0, split, kt0, nkt);
                for (int i = 0; i < nkt; i++, it++) {
                    const int s = it % a.n_tma;
                    const uint32_t ph = (uint32_t)(it / a.n_tma) & 1u;
                    if (!gm_wait(&empty[s], ph ^ 1u)) { atomicCAS(a.err, 0, 11); ok = false; break; }
                    uint8_t *st = gsm + (size_t)s * stage_bytes;
                    mbar_arrive_expect_tx(&full[s], stage_bytes);
                    const int kx = (kt0 + i) * a.bk;
                    tma_load_2d(st, &tm_w, kx, n0, &full[s]);
                    if (TF32) tma_load_2d(st + a_bytes, &tm_wl, kx, n0, &full[s]);
                    uint8_t *sb = st + a_bytes * a_parts;
                    tma_load_2d(sb, &tm_bh, kx, m0, &full[s]);
                    if (a.q8 || TF32) tma_load_2d(sb + b_bytes, &tm_bl, kx, m0, &full[s]);
                }
            }
            // every issued copy has landed before the CTA can finish
            for (int s = 0; s < a.n_tma; s++) {
                const int fills = it / a.n_tma + (it % a.n_tma > s ? 1 : 0);
                if (fills) gm_wait(&full[s], (uint32_t)(fills - 1) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            // D f32 (bits 4-5 = 1); A/B f16 (0) or tf32 (2) in bits 7-9 / 10-12;
            // K-major both; N >> 3 at bit 17, M >> 4 at bit 24
            const uint32_t fmt = TF32 ? 2u : 0u;
            const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
                                   ((uint32_t)(GM_BM >> 4) << 24);
            int it = 0, tc = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, tc++) {
                int n0, m0, split, kt0, nkt;
                coords(t, n0, m0, split, kt0, nkt);
                const int buf = tc & 1;
                if (!gm_wait(&tempty[buf], ((uint32_t)(tc >> 1) & 1u) ^ 1u)) { atomicCAS(a.err, 0, 15); break; }
                tc_fence_after();
                const uint32_t acc_t = tmem + (uint32_t)buf * acc_cols;
                for (int i = 0; i < nkt; i++, it++) {
                    const int s = it % a.n_tma;
                    const uint32_t ph = (uint32_t)(it / a.n_tma) & 1u;
                    const int c = it % a.n_conv;
                    const uint32_t cph = (uint32_t)(it / a.n_conv) & 1u;
                    if (!gm_wait(&full[s], ph) || (a.q8 && !gm_wait(&cfull[c], cph))) {
                        atomicCAS(a.err, 0, 12);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint8_t *st = gsm + (size_t)s * stage_bytes;
                    const uint8_t *ahi = a.q8 ? conv + (size_t)c * 32768 : st;
                    const uint8_t *alo = ahi + 16384;
                    const uint8_t *bhi = st + a_bytes * a_parts, *blo = bhi + b_bytes;
                    if constexpr (TF32) {
                        // four k-steps of 8 tf32 (32 bytes) per stage: hi*hi + hi*lo + lo*hi
#pragma unroll
                        // hi*hi accumulates apart from the two cross terms, which
                        // are 2^-11 smaller: the accumulator's own rounding then
                        // acts on the large sum once per k-step, not three times
                        for (int k = 0; k < 4; k++) {
                            const uint32_t acc = (i | k) != 0;
                            const uint32_t acc_s = acc_t + a.small_off;
                            umma_tf32(acc_t, sw128_desc(st + 32 * k), sw128_desc(bhi + 32 * k), idesc, acc);
                            umma_tf32(acc_s, sw128_desc(st + 32 * k), sw128_desc(blo + 32 * k), idesc, acc);
                            umma_tf32(acc_s, sw128_desc(st + a_bytes + 32 * k), sw128_desc(bhi + 32 * k), idesc, 1u);
                        }
                        umma_commit(&empty[s]);
                    } else {
#pragma unroll
                        for (int k = 0; k < GM_BK / 16; k++) {
                            const uint32_t acc = (i | k) != 0;
                            umma_f16(acc_t, sw128_desc(ahi + 32 * k), sw128_desc(bhi + 32 * k), idesc, acc);
                            if (a.q8) {
                                // the two cross terms (2^-11 of hi*hi) accumulate apart
                                const uint32_t acc_s = acc_t + a.small_off;
                                umma_f16(acc_s, sw128_desc(ahi + 32 * k), sw128_desc(blo + 32 * k), idesc, acc);
                                umma_f16(acc_s, sw128_desc(alo + 32 * k), sw128_desc(bhi + 32 * k), idesc, 1u);
                            }
                        }
                        umma_commit(&empty[s]);
                        if (a.q8) umma_commit(&cempty[c]);
                    }
                }
                umma_commit(&tfull[buf]);   // fires once this tile's MMAs have completed
            }
        }
    } else if (warp < 2 + GM_CONV_THREADS / 32) {
        // ------------------------------------------------ convert (Q8_0)
        // thread t converts the 16-byte pieces t and t + 256 of the raw
        // tile (row i/4, values 16*(i%4) .. +16: half of Q8_0 block
        // (i%4)/2), so a warp reads 512 consecutive bytes (no bank
        // conflicts) and writes whole swizzled 16-byte chunks.
        if (a.q8) {
            const int t = threadIdx.x - 64;
            const int kb_total = a.K / 32;
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                int n0, m0, split, kt0, nkt;
                coords(tile, n0, m0, split, kt0, nkt);
                int rr[2], qq[2];
                const uint16_t *scp[2];
                bool rv[2];
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const int i = t + 256 * u;
                    rr[u] = i >> 2;
                    qq[u] = i & 3;
                    rv[u] = n0 + rr[u] < a.N;
                    scp[u] = a.sc + (int64_t)(rv[u] ? n0 + rr[u] : 0) * kb_total + (qq[u] >> 1);
                }
                for (int i = 0; i < nkt; i++, it++) {
                    const int s = it % a.n_tma;
                    const uint32_t ph = (uint32_t)(it / a.n_tma) & 1u;
                    const int c = it % a.n_conv;
                    const uint32_t cph = (uint32_t)(it / a.n_conv) & 1u;
                    uint16_t dh[2];
#pragma unroll
                    for (int u = 0; u < 2; u++) dh[u] = rv[u] ? __ldg(scp[u] + (kt0 + i) * 2) : (uint16_t)0;
                    const bool okf = gm_wait(&full[s], ph), okc = gm_wait(&cempty[c], cph ^ 1u);
                    if (!okf || !okc) { atomicCAS(a.err, 0, 13); ok = false; break; }
                    const int4 *src = reinterpret_cast<const int4 *>(gsm + (size_t)s * stage_bytes);
                    int4 raw[2];
#pragma unroll
                    for (int u = 0; u < 2; u++) raw[u] = src[t + 256 * u];
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        uint8_t *hi = conv + (size_t)c * 32768 + rr[u] * 128;
                        uint8_t *lo = hi + 16384;
                        const __half2 d2 = __half2half2(__ushort_as_half(dh[u]));   // the fp16 scale itself
                        const uint32_t w4[4] = {(uint32_t)raw[u].x, (uint32_t)raw[u].y, (uint32_t)raw[u].z,
                                                (uint32_t)raw[u].w};
#pragma unroll
                        for (int hc = 0; hc < 2; hc++) {   // two 8-value chunks
                            uint32_t h[4], l[4];
#pragma unroll
                            for (int e = 0; e < 2; e++) {
                                // 4 int8 -> two exact half2: bytes q+128 under exponent 0x64
                                // give 1152 + q, minus 1152 exactly
                                const uint32_t x = w4[2 * hc + e] ^ 0x80808080u;
                                const uint32_t p01 = __byte_perm(x, 0x64646464u, 0x5140);
                                const uint32_t p23 = __byte_perm(x, 0x64646464u, 0x7362);
                                const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));   // 1152
                                const __half2 q01 = __hsub2(*reinterpret_cast<const __half2 *>(&p01), bias);
                                const __half2 q23 = __hsub2(*reinterpret_cast<const __half2 *>(&p23), bias);
                                // hi = fp16(d*q) (one rounding of the exact product);
                                // lo = fp16(d*q - hi) (fused: exact remainder, one rounding)
                                const __half2 h01 = __hmul2(d2, q01), h23 = __hmul2(d2, q23);
                                const __half2 l01 = __hfma2(d2, q01, __hneg2(h01));
                                const __half2 l23 = __hfma2(d2, q23, __hneg2(h23));
                                h[2 * e] = *reinterpret_cast<const uint32_t *>(&h01);
                                h[2 * e + 1] = *reinterpret_cast<const uint32_t *>(&h23);
                                l[2 * e] = *reinterpret_cast<const uint32_t *>(&l01);
                                l[2 * e + 1] = *reinterpret_cast<const uint32_t *>(&l23);
                            }
                            const int chunk = (2 * qq[u] + hc) ^ (rr[u] & 7);   // 128-byte swizzle
                            *reinterpret_cast<uint4 *>(hi + chunk * 16) = make_uint4(h[0], h[1], h[2], h[3]);
                            *reinterpret_cast<uint4 *>(lo + chunk * 16) = make_uint4(l[0], l[1], l[2], l[3]);
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor core
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&cfull[c]);
                }
            }
        }
    } else {
        // -------------------------------------------------------- epilogue
        // warp w reads TMEM lanes 32*(w%4) .. +32 (weight rows) of the
        // accumulator; the MMAs of the next tile run into the other one.
        const int et = threadIdx.x - (2 + GM_CONV_THREADS / 32) * 32;
        const int q = warp & 3;
        int tc = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, tc++) {
            int n0, m0, split, kt0, nkt;
            coords(tile, n0, m0, split, kt0, nkt);
            const int buf = tc & 1;
            const bool okt = gm_wait(&tfull[buf], (uint32_t)(tc >> 1) & 1u);
            tc_fence_after();
            const int r = q * 32 + lane, n = n0 + r;
            const bool split_k = a.splits > 1;
            if (!okt) atomicCAS(a.err, 0, 14);
            for (int j = 0; okt && j * 16 < BN; j++) {
                uint32_t v[16];
                const uint32_t ta = tmem + (uint32_t)buf * acc_cols + ((uint32_t)(q * 32) << 16) + (uint32_t)(j * 16);
                tmem_ld16(ta, v);
                if (TF32 || a.q8) {
                    uint32_t w[16];
                    tmem_ld16(ta + a.small_off, w);
#pragma unroll
                    for (int e = 0; e < 16; e++)
                        v[e] = __float_as_uint(__fadd_rn(__uint_as_float(v[e]), __uint_as_float(w[e])));
                }
                if (n < a.N) {
                    if (split_k) {
                        // partials [split][N][Mp], this thread's 16 columns contiguous
                        float4 *pw =
                            reinterpret_cast<float4 *>(a.ws + ((int64_t)split * a.N + n) * a.Mp + m0 + j * 16);
#pragma unroll
                        for (int q4 = 0; q4 < 4; q4++)
                            pw[q4] = make_float4(__uint_as_float(v[4 * q4]), __uint_as_float(v[4 * q4 + 1]),
                                                 __uint_as_float(v[4 * q4 + 2]), __uint_as_float(v[4 * q4 + 3]));
                    } else {
                        gm_store<TF32>(a, m0 + j * 16, n, reinterpret_cast<const float *>(v));
                    }
                }
            }
            // the accumulator is free for the tile after next
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            if (split_k) {
                // the last CTA of this tile adds the split partials in split order
                asm volatile("bar.sync 2, %0;" ::"r"(GM_EPI_THREADS) : "memory");
                if (et == 0) {
                    fence_acq_rel_gpu();
                    const unsigned tid = (unsigned)(tile / a.splits);
                    s_last = atomicAdd(a.cnt + tid, 1u) == (unsigned)(a.splits - 1);
                    if (s_last) {
                        fence_acq_rel_gpu();
                        a.cnt[tid] = 0;   // ready for the next launch
                    }
                }
                asm volatile("bar.sync 2, %0;" ::"r"(GM_EPI_THREADS) : "memory");
                if (s_last && n < a.N) {
                    // 16 columns x 2 splits (8 vector loads) in flight at a
                    // time; the sums still run in split order
#pragma unroll 1
                    for (int j = 0; j * 16 < BN; j++) {
                        float4 acc[4];
#pragma unroll
                        for (int q4 = 0; q4 < 4; q4++) acc[q4] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
                        for (int s0 = 0; s0 < a.splits; s0 += 2) {
                            float4 vv[2][4];
#pragma unroll
                            for (int u = 0; u < 2; u++) {
                                const float4 *pr = reinterpret_cast<const float4 *>(
                                    a.ws + ((int64_t)(s0 + u) * a.N + n) * a.Mp + m0 + j * 16);
#pragma unroll
                                for (int q4 = 0; q4 < 4; q4++)
                                    vv[u][q4] = s0 + u < a.splits ? __ldcg(pr + q4) : make_float4(0.f, 0.f, 0.f, 0.f);
                            }
#pragma unroll
                            for (int u = 0; u < 2; u++)
                                if (s0 + u < a.splits)
#pragma unroll
                                    for (int q4 = 0; q4 < 4; q4++) {
                                        acc[q4].x = __fadd_rn(acc[q4].x, vv[u][q4].x);
                                        acc[q4].y = __fadd_rn(acc[q4].y, vv[u][q4].y);
                                        acc[q4].z = __fadd_rn(acc[q4].z, vv[u][q4].z);
                                        acc[q4].w = __fadd_rn(acc[q4].w, vv[u][q4].w);
                                    }
                        }
                        gm_store<TF32>(a, m0 + j * 16, n, reinterpret_cast<const float *>(acc));
                    }
                }
                asm volatile("bar.sync 2, %0;" ::"r"(GM_EPI_THREADS) : "memory");   // s_last reused next tile
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
    }
}

// Emits 8 consecutive activation values (row offset o) as the GEMM operand:
// Q8_0 -> (hi, lo) fp16 of the dequantised block values (quantisation
// bit-exact with the GEMV path's, rule `rule`; the four threads of a 32-value
// block are consecutive lanes and all take part in the shuffles); F16 ->
// fp16(x).
__device__ __forceinline__ void act_emit8(const float (&v)[8], bool valid, int64_t o, int q8, int rule, __half *bh,
                                          __half *bl) {
    if (!q8) {
        if (valid) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                w[j] = (uint32_t)__half_as_ushort(__float2half_rn(v[2 * j])) |
                       ((uint32_t)__half_as_ushort(__float2half_rn(v[2 * j + 1])) << 16);
            *reinterpret_cast<uint4 *>(bh + o) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        return;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const uint16_t dh = f2h(d);
    const bool x86 = rule == VB_QRULE_X86;
    float id;
    if (x86) id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    const float df = h2f(dh);
    uint32_t wh[4], wl[4];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float t = __fmul_rn(v[j], id);
        const int q = x86 ? __float2int_rn(t) : (int)roundf(t);
        const float dv = __fmul_rn(df, (float)q);
        const __half h = __float2half_rn(dv);
        const __half l = __float2half_rn(__fsub_rn(dv, __half2float(h)));
        if (j & 1) {
            wh[j >> 1] |= (uint32_t)__half_as_ushort(h) << 16;
            wl[j >> 1] |= (uint32_t)__half_as_ushort(l) << 16;
        } else {
            wh[j >> 1] = __half_as_ushort(h);
            wl[j >> 1] = __half_as_ushort(l);
        }
    }
    if (valid) {
        *reinterpret_cast<uint4 *>(bh + o) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
        *reinterpret_cast<uint4 *>(bl + o) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
    }
}

__device__ __forceinline__ void load8(const float *p, bool vec, float (&v)[8]) {
    if (vec) {
        const float4 a0 = *reinterpret_cast<const float4 *>(p), a1 = *reinterpret_cast<const float4 *>(p + 4);
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = p[j];
    }
}

// Activation operand(s), one thread per 8 values; row m reads x row
// (m % x_mod).  vec: x rows are 16-byte aligned (float4 loads).  With
// swiglu_f > 0 the x rows are [gate (F) | up (F)] and the operand is the
// SwiGLU middle of vcpm_mlp, bf16(bf16(silu(bf16 g)) * bf16 u)
// (src/minicpm4.c:441-456, the swiglu_rows_kernel formula), so the
// down-projection reads the gate/up output directly.
__global__ void gemm_act_kernel(const float *x, int64_t ldx, int64_t x_mod, int M, int K, int q8, int rule, int vec,
                                int swiglu_f, __half *bh, __half *bl) {
    pdl_trigger();
    pdl_wait();
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // item of 8 values
    const int ipr = K >> 3;
    const bool valid = e < (int64_t)M * ipr;
    const int m = valid ? (int)(e / ipr) : 0, k0 = valid ? (int)(e - (int64_t)m * ipr) * 8 : 0;
    const float *xr = x + (int64_t)(m % x_mod) * ldx + k0;
    float v[8];
    load8(xr, vec, v);
    if (swiglu_f > 0) {
        float u[8];
        load8(xr + swiglu_f, vec, u);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = bf16r(__fmul_rn(bf16r(silu_f(bf16r(v[j]))), bf16r(u[j])));
    }
    act_emit8(v, valid, (int64_t)m * K + k0, q8, rule, bh, bl);
}

// The operand of a mat-mul that follows vcpm_rms_norm with a weight and
// bf16 rounding (src/minicpm4.c:132-152): one CTA per row computes the row
// statistic as rms_norm_kernel does (fp32 squares summed in double, mean
// rounded to fp32, 1/sqrt(mean + eps)), then each value
// bf16(bf16(x * scale) * w) goes straight into the operand.  K <= 8 * 256 *
// ACT_NORM_ITEMS.
constexpr int ACT_NORM_THREADS = 256, ACT_NORM_ITEMS = 4;

__global__ void __launch_bounds__(ACT_NORM_THREADS) gemm_act_norm_kernel(const float *x, int64_t ldx, int64_t x_mod,
                                                                          int K, int q8, int rule, int vec,
                                                                          const float *__restrict__ nw, float eps,
                                                                          __half *bh, __half *bl) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    const float *xr = x + (int64_t)(m % x_mod) * ldx;
    const int ipr = K >> 3;
    float v[ACT_NORM_ITEMS][8];
    double s = 0.0;
#pragma unroll
    for (int it = 0; it < ACT_NORM_ITEMS; it++) {
        const int item = it * ACT_NORM_THREADS + threadIdx.x;
        if (item < ipr) {
            load8(xr + item * 8, vec, v[it]);
#pragma unroll
            for (int j = 0; j < 8; j++) s += (double)__fmul_rn(v[it][j], v[it][j]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) v[it][j] = 0.0f;
        }
    }
    __shared__ double red[ACT_NORM_THREADS / 32];
    __shared__ float s_scale;
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < ACT_NORM_THREADS / 32 ? red[threadIdx.x] : 0.0;
        t = warp_sum_d(t);
        if (threadIdx.x == 0) {
            const float mean = __double2float_rn(__ddiv_rn(t, (double)K));
            s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        }
    }
    __syncthreads();
    const float scale = s_scale;
#pragma unroll
    for (int it = 0; it < ACT_NORM_ITEMS; it++) {
        const int item = it * ACT_NORM_THREADS + threadIdx.x;
        if (it * ACT_NORM_THREADS >= ipr) break;     // uniform over the CTA
        const bool valid = item < ipr;
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float wv = valid ? __ldg(nw + item * 8 + j) : 0.0f;
            y[j] = bf16r(__fmul_rn(bf16r(__fmul_rn(v[it][j], scale)), wv));
        }
        act_emit8(y, valid, (int64_t)m * K + (int64_t)(valid ? item : 0) * 8, q8, rule, bh, bl);
    }
}

// ============================================================ int8 path
// Q8_0 x Q8_0 on the integer tensor cores (tcgen05.mma kind::i8): the exact
// semantics of ggml's block dot,
//   y[m][n] = sum_b (d_w[n,b] * d_x[m,b]) * isum_b,  isum_b = sum_{j<32} qw qx,
// with isum_b an exact int32 for every (weight row, activation row) pair.
// The block scales differ per block, so integer sums cannot run across
// blocks: one MMA (K = 32) per Q8_0 block writes isum_b into one of four
// TMEM buffers, and the epilogue warps fold each buffer into fp32 registers
// as acc = fma(float(isum_b), d_w * d_x, acc) in block order (the product of
// two fp16 scales is exact in fp32).
//
// int32 -> fp32 without a conversion: every buffer is preset to the int32
// 0x4B400000 (the bits of 1.5 * 2^23) and the MMA accumulates into it, so
// a buffer word holds the bits of the fp32 1.5 * 2^23 + isum_b, exactly
// (|isum_b| <= 32 * 127 * 128 < 2^22); subtracting 1.5 * 2^23 is exact too.
// The epilogue reads a buffer, writes the preset back, and works on pairs
// of columns with the packed fp32 operations (add, mul, fma: each rounds
// as its scalar form does): 1.5 instructions per output and block.
//
// The weight's repacked int8 quants stream by TMA as they are; the
// activation is quantized once per call (gemm_act_i8_kernel) into int8
// rows and fp32 block scales stored transposed, [K/32][Mq], so a stage's
// scales are one TMA box.
//
// Tile: 128 weight rows (MMA M, TMEM lanes) x BN = NG * CW activation rows
// (MMA N, TMEM columns) x 128 k per stage (one 128-byte swizzle row = four
// blocks).  Warp 0 issues TMA, warp 1 allocates TMEM and issues the MMAs,
// warps 2 .. 4 * NG + 1 are the epilogue: warp w reads TMEM lanes
// 32*(w%4).. and columns [CW * g, CW * (g+1)) with g = (w-2)/4.  A stage is
// refilled once its MMAs have completed AND the epilogue has read its scales.
constexpr int GI_BK = 128;
constexpr int GI_MIN_M = 3;     // fewest activation rows routed to the int8 kernel (gemm_small_m)
// NG column groups of CW columns: BN = NG * CW, 4 * NG epilogue warps
constexpr int gi_threads(int ng) { return 64 + 128 * ng; }
constexpr int GI_DBUF = 4;
constexpr int GI_MAX_STAGES = 6;
constexpr uint32_t GI_MAGIC = 0x4B400000u;     // bits of 12582912.0f = 1.5 * 2^23

// D += A * B (D holds the preset)
__device__ __forceinline__ void umma_i8(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.eq.b32 p, 0, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc)
        : "memory");
}

// TMEM loads of CW columns of this warp's 32 lanes, with the wait in the
// same statement (see tmem_ld16)
template <int CW>
__device__ __forceinline__ void tmem_ld_cw(uint32_t taddr, uint32_t (&r)[CW]);
template <>
__device__ __forceinline__ void tmem_ld_cw<8>(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld_cw<16>(uint32_t taddr, uint32_t (&r)[16]) {
    tmem_ld16(taddr, r);
}
// Presets CW columns of this warp's 32 lanes to GI_MAGIC and waits for the
// stores.
template <int CW>
__device__ __forceinline__ void tmem_preset(uint32_t taddr) {
    const uint32_t m = GI_MAGIC;
    if constexpr (CW == 8) {
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};\n"
            "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
            "r"(m)
            : "memory");
    } else {
#pragma unroll
        for (int c = 0; c < CW; c += 16)
            asm volatile(
                "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
                    taddr + (uint32_t)c),
                "r"(m)
                : "memory");
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
}

template <int CW, int NG>
__global__ void __launch_bounds__(gi_threads(NG), 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_dx, const GemmArgs a) {
    constexpr int BN = NG * CW;
    constexpr int GI_EPI_WARPS = 4 * NG;
    extern __shared__ uint8_t gsm_raw[];
    uint8_t *gsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bars[2 * GI_MAX_STAGES + 2 * GI_DBUF];
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;
    uint64_t *full = bars, *empty = bars + GI_MAX_STAGES, *dfull = bars + 2 * GI_MAX_STAGES, *dempty = dfull + GI_DBUF;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t a_bytes = GM_BM * GI_BK;      // 16 KB of weight quants
    constexpr uint32_t b_bytes = BN * GI_BK;         // activation quants
    constexpr uint32_t s_bytes = 4u * BN * 4u;       // the four blocks' activation scales
    constexpr uint32_t stage_bytes = a_bytes + b_bytes + ((s_bytes + 1023) & ~1023u);
    const int n_tiles = a.tiles_n * a.tiles_m * a.splits;
    const uint32_t pcols = a.tmem_cols / GI_DBUF;
    const int nbk = a.K / QK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < GI_MAX_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + GI_EPI_WARPS);
        }
        for (int d = 0; d < GI_DBUF; d++) {
            mbar_init(&dfull[d], 1);
            mbar_init(&dempty[d], GI_EPI_WARPS);
        }
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int q = warp & 3, cg = (warp - 2) >> 2, c0 = cg * CW;
    if (warp >= 2) {
        // the preset of every buffer, before the first MMA
#pragma unroll 1
        for (int d = 0; d < GI_DBUF; d++)
            tmem_preset<CW>(tmem + (uint32_t)d * pcols + ((uint32_t)(q * 32) << 16) + (uint32_t)c0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_wait();
    pdl_trigger();

    auto coords = [&](int t, int &n0, int &m0, int &split, int &kt0, int &nkt) {
        split = t % a.splits;
        t /= a.splits;
        m0 = (t % a.tiles_m) * BN;
        n0 = (t / a.tiles_m) * GM_BM;
        kt0 = split * a.kt_per_split;
        nkt = min(a.kt_per_split, a.kt_total - kt0);
    };

    if (warp == 0) {
        // ------------------------------------------------------------ TMA
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                int n0, m0, split, kt0, nkt;
                coords(t, n0, m0, split, kt0, nkt);
                for (int i = 0; i < nkt; i++, it++) {
                    const int s = it % a.n_tma;
                    const uint32_t ph = (uint32_t)(it / a.n_tma) & 1u;
                    if (!gm_wait(&empty[s], ph ^ 1u)) { atomicCAS(a.err, 0, 21); ok = false; break; }
                    uint8_t *st = gsm + (size_t)s * stage_bytes;
                    mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes + s_bytes);
                    const int kx = (kt0 + i) * GI_BK;
                    tma_load_2d(st, &tm_w, kx, n0, &full[s]);
                    tma_load_2d(st + a_bytes, &tm_x, kx, m0, &full[s]);
                    tma_load_2d(st + a_bytes + b_bytes, &tm_dx, m0, kx / QK, &full[s]);
                }
            }
            for (int s = 0; s < a.n_tma; s++) {
                const int fills = it / a.n_tma + (it % a.n_tma > s ? 1 : 0);
                if (fills) gm_wait(&full[s], (uint32_t)(fills - 1) & 1u);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            // D s32 (bits 4-5 = 2); A and B signed 8-bit (1) in bits 7-9 / 10-12;
            // K-major both; N >> 3 at bit 17, M >> 4 at bit 24
            const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                   ((uint32_t)(GM_BM >> 4) << 24);
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                int n0, m0, split, kt0, nkt;
                coords(t, n0, m0, split, kt0, nkt);
                for (int i = 0; i < nkt && ok; i++, it++) {
                    const int s = it % a.n_tma;
                    const uint32_t ph = (uint32_t)(it / a.n_tma) & 1u;
                    if (!gm_wait(&full[s], ph)) { atomicCAS(a.err, 0, 22); ok = false; break; }
                    uint8_t *st = gsm + (size_t)s * stage_bytes;
                    // block k of every stage goes to buffer k (four blocks per
                    // stage), so the buffers turn over once per stage
                    const uint32_t bph = (uint32_t)it & 1u;
#pragma unroll
                    for (int k = 0; k < GI_DBUF; k++) {
                        if (!gm_wait(&dempty[k], bph ^ 1u)) { atomicCAS(a.err, 0, 23); ok = false; break; }
                        tc_fence_after();
                        umma_i8(tmem + (uint32_t)k * pcols, sw128_desc(st + 32 * k), sw128_desc(st + a_bytes + 32 * k),
                                idesc);
                        umma_commit(&dfull[k]);
                    }
                    umma_commit(&empty[s]);   // the stage's MMAs are done with its operands
                }
            }
        }
    } else {
        // -------------------------------------------------------- epilogue
        const int et = threadIdx.x - 64;
        const float2 nmagic = make_float2(-12582912.0f, -12582912.0f);
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            int n0, m0, split, kt0, nkt;
            coords(tile, n0, m0, split, kt0, nkt);
            const int r = q * 32 + lane, n = n0 + r;
            const bool nv = n < a.N;
            const uint2 *scp = reinterpret_cast<const uint2 *>(a.sc + (int64_t)(nv ? n : 0) * nbk) + kt0;
            float2 acc[CW / 2];
#pragma unroll
            for (int c = 0; c < CW / 2; c++) acc[c] = make_float2(0.0f, 0.0f);
            // the four weight scales of a stage: one 8-byte load (K % 128 == 0),
            // fetched a stage ahead
            uint2 dw_next = nv ? __ldg(scp) : make_uint2(0u, 0u);
            for (int i = 0; i < nkt; i++, it++) {
                const int s = it % a.n_tma;
                const uint32_t ph = (uint32_t)(it / a.n_tma) & 1u;
                const uint32_t bph = (uint32_t)it & 1u;   // the buffers turn over once per stage
                const uint2 dw4 = dw_next;
                if (i + 1 < nkt && nv) dw_next = __ldg(scp + i + 1);
                const float2 dw01 = __half22float2(*reinterpret_cast<const __half2 *>(&dw4.x));
                const float2 dw23 = __half22float2(*reinterpret_cast<const __half2 *>(&dw4.y));
                if (ok && !gm_wait(&full[s], ph)) { atomicCAS(a.err, 0, 24); ok = false; }
                const float4 *dx4 =
                    reinterpret_cast<const float4 *>(gsm + (size_t)s * stage_bytes + a_bytes + b_bytes) + c0 / 4;
#pragma unroll
                for (int k = 0; k < GI_DBUF; k++) {
                    if (ok && !gm_wait(&dfull[k], bph)) { atomicCAS(a.err, 0, 25); ok = false; }
                    tc_fence_after();
                    const float dw = k == 0 ? dw01.x : k == 1 ? dw01.y : k == 2 ? dw23.x : dw23.y;
                    const float2 dw2 = make_float2(dw, dw);
                    const uint32_t tb = tmem + (uint32_t)k * pcols + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
                    // in loads of at most 16 columns (registers: 16 epilogue warps)
                    constexpr int LC = CW < 16 ? CW : 16;
#pragma unroll
                    for (int c = 0; c < CW; c += LC) {
                        uint32_t v[LC];
                        tmem_ld_cw<LC>(tb + (uint32_t)c, v);
                        if (c + LC == CW) {
                            // the buffer is read: preset it and hand it back to the MMA
                            tmem_preset<CW>(tb);
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&dempty[k]);
                        }
#pragma unroll
                        for (int e = 0; e < LC / 4; e++) {
                            const float4 dx = dx4[k * (BN / 4) + c / 4 + e];
                            const int o = c / 2 + 2 * e;
                            acc[o] = __ffma2_rn(
                                __fadd2_rn(make_float2(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1])), nmagic),
                                __fmul2_rn(dw2, make_float2(dx.x, dx.y)), acc[o]);
                            acc[o + 1] = __ffma2_rn(
                                __fadd2_rn(make_float2(__uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3])),
                                           nmagic),
                                __fmul2_rn(dw2, make_float2(dx.z, dx.w)), acc[o + 1]);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);   // this warp has read the stage's scales
            }
            // ---- output (or split partials) for row n, columns m0 + c0 ..
            const bool split_k = a.splits > 1;
            const float *accf = reinterpret_cast<const float *>(acc);
            if (nv) {
                if (split_k) {
                    float4 *pw = reinterpret_cast<float4 *>(a.ws + ((int64_t)split * a.N + n) * a.Mp + m0 + c0);
#pragma unroll
                    for (int q4 = 0; q4 < CW / 4; q4++)
                        pw[q4] = make_float4(accf[4 * q4], accf[4 * q4 + 1], accf[4 * q4 + 2], accf[4 * q4 + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < CW; j += 8) gm_store8(a, m0 + c0 + j, n, accf + j);
                }
            }
            if (split_k) {
                // the last CTA of this tile adds the split partials in split order
                asm volatile("bar.sync 2, %0;" ::"r"(32 * GI_EPI_WARPS) : "memory");
                if (et == 0) {
                    fence_acq_rel_gpu();
                    const unsigned tid = (unsigned)(tile / a.splits);
                    s_last = atomicAdd(a.cnt + tid, 1u) == (unsigned)(a.splits - 1);
                    if (s_last) {
                        fence_acq_rel_gpu();
                        a.cnt[tid] = 0;
                    }
                }
                asm volatile("bar.sync 2, %0;" ::"r"(32 * GI_EPI_WARPS) : "memory");
                if (s_last && nv) {
#pragma unroll 1
                    for (int j = 0; j < CW; j += 8) {
                        float4 sum[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll 1
                        for (int sp = 0; sp < a.splits; sp++) {
                            const float4 *pr = reinterpret_cast<const float4 *>(
                                a.ws + ((int64_t)sp * a.N + n) * a.Mp + m0 + c0 + j);
#pragma unroll
                            for (int q4 = 0; q4 < 2; q4++) {
                                const float4 v = __ldcg(pr + q4);
                                sum[q4].x = __fadd_rn(sum[q4].x, v.x);
                                sum[q4].y = __fadd_rn(sum[q4].y, v.y);
                                sum[q4].z = __fadd_rn(sum[q4].z, v.z);
                                sum[q4].w = __fadd_rn(sum[q4].w, v.w);
                            }
                        }
                        gm_store8(a, m0 + c0 + j, n, reinterpret_cast<const float *>(sum));
                    }
                }
                asm volatile("bar.sync 2, %0;" ::"r"(32 * GI_EPI_WARPS) : "memory");
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
    }
}

// Q8_0 quantization of 8 activation values (ggml's rule, bit-exact; the four
// threads of a 32-value block are consecutive lanes and all take part in the
// shuffles) into the int8 operand row and the transposed scale table.
__device__ __forceinline__ void act_emit8_i8(const float (&v)[8], bool valid, int m, int k0, int K, int Mp, int rule,
                                             int8_t *qx, float *dxt) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const uint16_t dh = f2h(d);
    const bool x86 = rule == VB_QRULE_X86;
    float id;
    if (x86) id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float t = __fmul_rn(v[j], id);
        const int qv = x86 ? __float2int_rn(t) : (int)roundf(t);
        w[j >> 2] |= ((uint32_t)(qv & 0xff)) << (8 * (j & 3));
    }
    if (valid) {
        *reinterpret_cast<uint2 *>(qx + (int64_t)m * K + k0) = make_uint2(w[0], w[1]);
        if ((k0 & 31) == 0) dxt[(int64_t)(k0 >> 5) * Mp + m] = h2f(dh);
    }
}

__global__ void gemm_act_i8_kernel(const float *x, int64_t ldx, int64_t x_mod, int M, int K, int Mp, int rule, int vec,
                                   int swiglu_f, int8_t *qx, float *dxt) {
    pdl_trigger();
    pdl_wait();
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // item of 8 values
    const int ipr = K >> 3;
    const bool valid = e < (int64_t)M * ipr;
    const int m = valid ? (int)(e / ipr) : 0, k0 = valid ? (int)(e - (int64_t)m * ipr) * 8 : 0;
    const float *xr = x + (int64_t)(m % x_mod) * ldx + k0;
    float v[8];
    load8(xr, vec, v);
    if (swiglu_f > 0) {
        float u[8];
        load8(xr + swiglu_f, vec, u);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = bf16r(__fmul_rn(bf16r(silu_f(bf16r(v[j]))), bf16r(u[j])));
    }
    act_emit8_i8(v, valid, m, k0, K, Mp, rule, qx, dxt);
}

// The int8 operand of a mat-mul that follows vcpm_rms_norm (the statistic
// and rounding of gemm_act_norm_kernel).
__global__ void __launch_bounds__(ACT_NORM_THREADS) gemm_act_i8_norm_kernel(const float *x, int64_t ldx, int64_t x_mod,
                                                                             int K, int Mp, int rule, int vec,
                                                                             const float *__restrict__ nw, float eps,
                                                                             int8_t *qx, float *dxt) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    const float *xr = x + (int64_t)(m % x_mod) * ldx;
    const int ipr = K >> 3;
    float v[ACT_NORM_ITEMS][8];
    double s = 0.0;
#pragma unroll
    for (int it = 0; it < ACT_NORM_ITEMS; it++) {
        const int item = it * ACT_NORM_THREADS + threadIdx.x;
        if (item < ipr) {
            load8(xr + item * 8, vec, v[it]);
#pragma unroll
            for (int j = 0; j < 8; j++) s += (double)__fmul_rn(v[it][j], v[it][j]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) v[it][j] = 0.0f;
        }
    }
    __shared__ double red[ACT_NORM_THREADS / 32];
    __shared__ float s_scale;
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < ACT_NORM_THREADS / 32 ? red[threadIdx.x] : 0.0;
        t = warp_sum_d(t);
        if (threadIdx.x == 0) {
            const float mean = __double2float_rn(__ddiv_rn(t, (double)K));
            s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        }
    }
    __syncthreads();
    const float scale = s_scale;
#pragma unroll
    for (int it = 0; it < ACT_NORM_ITEMS; it++) {
        const int item = it * ACT_NORM_THREADS + threadIdx.x;
        if (it * ACT_NORM_THREADS >= ipr) break;     // uniform over the CTA
        const bool valid = item < ipr;
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float wv = valid ? __ldg(nw + item * 8 + j) : 0.0f;
            y[j] = bf16r(__fmul_rn(bf16r(__fmul_rn(v[it][j], scale)), wv));
        }
        act_emit8_i8(y, valid, m, valid ? item * 8 : 0, K, Mp, rule, qx, dxt);
    }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D tensor map over a row-major [rows][cols] array of `esize`-byte
// elements, box [box_rows][box_cols].
static bool make_map(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int esize, int64_t cols, int64_t rows,
                     int box_cols, int box_rows, bool swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * esize)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct ActMaps {                // TMA descriptors of one activation buffer shape
    const void *bh = nullptr, *bl = nullptr;
    int K = 0, M = 0, BN = 0;
    bool tf32 = false, i8 = false;
    CUtensorMap th, tl;
};

struct GemmState {
    Arena act;                  // activation operands
    Arena part;                 // split partials
    unsigned *cnt = nullptr;    // tile counters
    int *err = nullptr;
    bool init = false;
    ActMaps cache[8];           // most recent activation descriptors
    int next = 0;
};

static GemmState *gemm_state(vb_ctx *ctx) {
    GemmState *g = static_cast<GemmState *>(ctx->gemm);
    if (g) return g;
    g = new GemmState();
    if (cudaMalloc(&g->cnt, 65536 * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(g->cnt, 0, 65536 * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&g->err, sizeof(int)) != cudaSuccess || cudaMemset(g->err, 0, sizeof(int)) != cudaSuccess) {
        cudaFree(g->cnt);
        cudaFree(g->err);
        delete g;
        return nullptr;
    }
    g->init = true;
    ctx->gemm = g;
    return g;
}

void gemm_free(vb_ctx *ctx) {
    GemmState *g = static_cast<GemmState *>(ctx->gemm);
    if (!g) return;
    cudaFree(g->act.ptr);
    cudaFree(g->part.ptr);
    cudaFree(g->cnt);
    cudaFree(g->err);
    delete g;
    ctx->gemm = nullptr;
}

int init_gemm(vb_ctx *ctx) {
    VB_CHECK(ctx, cudaFuncSetAttribute(gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GM_SMEM_BUDGET + 1024));
    VB_CHECK(ctx, cudaFuncSetAttribute(gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GM_SMEM_BUDGET + 1024));
    VB_CHECK(ctx, cudaFuncSetAttribute(gemm_i8_kernel<8, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GM_SMEM_BUDGET + 1024));
    VB_CHECK(ctx, cudaFuncSetAttribute(gemm_i8_kernel<8, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GM_SMEM_BUDGET + 1024));
    VB_CHECK(ctx, cudaFuncSetAttribute(gemm_i8_kernel<16, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GM_SMEM_BUDGET + 1024));
    VB_CHECK(ctx, cudaFuncSetAttribute(gemm_i8_kernel<32, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GM_SMEM_BUDGET + 1024));
    // the mat-mul kernels' counters and error word exist from creation on, so
    // no later call allocates them (and every call can be captured)
    if (!gemm_state(ctx)) return set_error(ctx, VB_ERR_OOM, "mat-mul state allocation failed");
    return VB_OK;
}

// Launch with programmatic stream serialization (the kernel begins with
// pdl_wait before it reads anything the previous kernel wrote).
template <typename... KArgs, typename... Args>
static cudaError_t pdl_launch(vb_ctx *ctx, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Q8_0 weights on the int8 tensor cores (gemm_i8_kernel); K % 128 == 0.
static int launch_gemm_i8(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, int64_t x_mod,
                          const MatmulOut &out, const GemmPro *pro) {
    GemmState *gs = gemm_state(ctx);
    if (!gs) return set_error(ctx, VB_ERR_OOM, "gemm: state allocation failed");
    const int K = (int)w->K, N = (int)w->N;
    const int tiles_n = (N + GM_BM - 1) / GM_BM;
    const int mr = (int)((M + 15) / 16 * 16);
    const int kt_total = K / GI_BK;
    // Tile width and K split: the epilogue (four fp32 operations per output
    // and Q8_0 block) sets a unit's time, ~ BN x k-stages + a fixed
    // per-unit cost, over waves of the persistent grid, plus the split
    // reduction (the last CTA of a tile reads every split's partials).
    int BN = 0, splits = 1;
    double best = 1e300;
    // (BN = 96: three column groups of 32, twelve epilogue warps -- with 4
    // groups of 32 the register budget of 16 epilogue warps spills)
    // (BN = 16, two column groups of 8, for M <= 16 only: the narrowest
    // MMA, half the epilogue warps of BN = 32 and no fold of absent rows)
    for (int cand : {96, 64, 32, 16}) {
        if (cand == 16 && mr > 16) continue;
        if (cand > 32 && cand > mr && (cand == 96 ? 64 : cand >> 1) >= mr) continue;
        const int64_t tiles = (int64_t)tiles_n * ((M + cand - 1) / cand);
        for (int sp = 1; sp <= std::max(1, kt_total / 2); sp++) {
            const int kps = (kt_total + sp - 1) / sp;
            const int64_t units = tiles * ((kt_total + kps - 1) / kps);
            const int64_t waves = (units + ctx->sm_count - 1) / ctx->sm_count;
            // split price: the last CTA of a tile adds every split's partials
            // (measured on B200 for M = 8 .. 704: 1 x splits x BN picks the
            // fastest tile and split of every swept shape)
            const double t = (double)waves * ((double)cand * kps + 256.0) + (sp > 1 ? 1.0 * sp * cand : 0.0);
            if (t < best * 0.999) { best = t; BN = cand; splits = sp; }
            if (units >= 4 * ctx->sm_count) break;
        }
    }
    if (BN == 0) {
        BN = 64;
        splits = 1;
    }
    const int tiles_m = (int)((M + BN - 1) / BN);
    const int tiles = tiles_m * tiles_n;
    const int kt_per_split = (kt_total + splits - 1) / splits;
    splits = (kt_total + kt_per_split - 1) / kt_per_split;
    if (tiles > 65536) return set_error(ctx, VB_ERR_INVALID_ARG, "gemm: too many tiles");

    const size_t stage = (size_t)GM_BM * GI_BK + (size_t)BN * GI_BK + (((size_t)16 * BN + 1023) & ~(size_t)1023);
    const int n_tma = (int)std::min<size_t>(GI_MAX_STAGES, GM_SMEM_BUDGET / stage);
    if (n_tma < 2) return set_error(ctx, VB_ERR_INVALID_ARG, "gemm: tile does not fit shared memory");
    const size_t smem = (size_t)n_tma * stage + 1024;
    uint32_t pcols = 32;
    while (pcols < (uint32_t)BN) pcols <<= 1;
    const uint32_t cols = GI_DBUF * pcols;

    // activation operand: int8 rows [M][K] and block scales [K/32][Mq]
    const int Mq = (int)((M + 3) / 4 * 4);
    const size_t qb = ((size_t)M * K + 1023) & ~(size_t)1023;
    int rc = arena_reserve(ctx, gs->act, qb + (size_t)(K / QK) * Mq * 4 + 512);
    if (rc) return rc;
    int8_t *qx = (int8_t *)gs->act.ptr;
    float *dxt = (float *)((uint8_t *)gs->act.ptr + qb);
    {
        const int64_t items = M * (K / 8);
        const int64_t lx = ldx ? ldx : (pro && pro->swiglu_f ? 2 * (int64_t)K : K);
        const int vec = ((uintptr_t)x % 16 == 0) && (lx % 4 == 0);
        const int64_t xm = x_mod > 0 ? x_mod : M;
        if (pro && pro->norm_w) {
            if (K > 8 * ACT_NORM_THREADS * ACT_NORM_ITEMS)
                return set_error(ctx, VB_ERR_INVALID_ARG, "gemm: fused RMSNorm row of %d values is too wide", K);
            VB_CHECK(ctx, pdl_launch(ctx, gemm_act_i8_norm_kernel, dim3((unsigned)M), dim3(ACT_NORM_THREADS), 0, x, lx,
                                     xm, K, Mq, ctx->qrule, vec, pro->norm_w, pro->eps, qx, dxt));
        } else {
            VB_CHECK(ctx, pdl_launch(ctx, gemm_act_i8_kernel, dim3((unsigned)((items + 255) / 256)), dim3(256), 0, x,
                                     lx, xm, (int)M, K, Mq, ctx->qrule, vec, pro ? pro->swiglu_f : 0, qx, dxt));
        }
        VB_LAUNCH_CHECK(ctx, "gemm_act_i8");
    }
    if (!w->tmap_i8_ok) {
        CUtensorMap *tw = reinterpret_cast<CUtensorMap *>(w->tmap_i8);
        w->tmap_i8_ok = make_map(tw, w->data, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, GI_BK, GM_BM, true);
        if (!w->tmap_i8_ok) return set_error(ctx, VB_ERR_BACKEND, "gemm: weight tensor map encoding failed");
    }
    // activation descriptors per (buffer, shape): th over the quants, tl over the scales
    ActMaps *am = nullptr;
    for (ActMaps &c : gs->cache)
        if (c.bh == qx && c.bl == dxt && c.K == K && c.M == (int)M && c.BN == BN && c.i8) am = &c;
    if (!am) {
        am = &gs->cache[gs->next];
        gs->next = (gs->next + 1) % 8;
        am->bh = nullptr;
        if (!make_map(&am->th, qx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, GI_BK, BN, true) ||
            !make_map(&am->tl, dxt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Mq, K / QK, BN, GI_BK / QK, false))
            return set_error(ctx, VB_ERR_BACKEND, "gemm: activation tensor map encoding failed");
        am->bh = qx;
        am->bl = dxt;
        am->K = K;
        am->M = (int)M;
        am->BN = BN;
        am->tf32 = false;
        am->i8 = true;
    }

    GemmArgs g{};
    g.q8 = 1;
    g.bk = GI_BK;
    g.K = K;
    g.N = N;
    g.M = (int)M;
    g.BN = BN;
    g.kt_total = kt_total;
    g.kt_per_split = kt_per_split;
    g.splits = splits;
    g.tiles_m = tiles_m;
    g.tiles_n = tiles_n;
    g.n_tma = n_tma;
    g.tmem_cols = cols;
    g.sc = w->scales;
    g.y = out.y;
    g.bias = out.bias;
    g.flags = out.flags;
    g.res = out.res;
    g.res_scale = out.res_scale;
    g.ldy = out.ldy ? out.ldy : N;
    g.seg = out.seg ? out.seg : M;
    g.seg_stride = out.seg ? out.seg_stride : 0;
    g.seg_off = out.seg ? out.seg_off : 0;
    g.seg_plain = g.seg >= M && g.seg_off == 0;
    g.cnt = gs->cnt;
    g.err = gs->err;
    if (splits > 1) {
        g.Mp = tiles_m * BN;
        rc = arena_reserve(ctx, gs->part, (size_t)splits * N * g.Mp * 4);
        if (rc) return rc;
        g.ws = (float *)gs->part.ptr;
    }
    const int n_work = tiles * splits;
    const CUtensorMap &twm = *reinterpret_cast<const CUtensorMap *>(w->tmap_i8);
    void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const GemmArgs) =
        BN == 96 ? gemm_i8_kernel<32, 3>
                 : BN == 64 ? gemm_i8_kernel<16, 4> : BN == 32 ? gemm_i8_kernel<8, 4> : gemm_i8_kernel<8, 2>;
    const int threads = gi_threads(BN == 96 ? 3 : BN == 16 ? 2 : 4);
    VB_CHECK(ctx, pdl_launch(ctx, kern, dim3((unsigned)std::min(n_work, ctx->sm_count)), dim3(threads), smem, twm,
                             am->th, am->tl, g));
    VB_LAUNCH_CHECK(ctx, "gemm_i8");
    return VB_OK;
}

// Where the int8 kernel beats the fp16 split kernel (B200 sweep of the
// MiniCPM4 and LocDiT projection shapes, M = 128 .. 1408): its epilogue work
// grows with M x N x K/32 while the split kernel's fixed per-call cost falls
// away, and the split kernel is weakest on long-K, narrow-N shapes.
static bool gemm_i8_faster(int64_t M, int64_t K, int64_t N) {
    return M <= 256 || (K >= 3 * N && M <= 1536) || (double)M * (double)N * (double)K <= 3.3e9;
}

// 3 <= M < 16 activation rows (decode steps of a few utterances) on the
// tensor cores with a 16-row tile (the absent rows zero-filled by TMA and
// never stored): Q8_0 on the int8 kernel, F16 on the kind::f16 kernel.
// Each streams every weight once at the tensor cores' pace, where the
// M <= 8 weight-streaming op and the GEMV kernels pay per activation row
// (B200, 28-layer Q8_0 decode step: M = 8 9.0 ms per token on those,
// 2.8 ms on the int8 kernel).
bool gemm_small_m(const vb_ctx *ctx, vb_weight w, int64_t M) {
    if (M < GI_MIN_M || M >= 16 || encode_fn() == nullptr) return false;
    if (w->type == VB_TYPE_Q8_0) return ctx->gemm_i8 != 0 && w->K % GI_BK == 0;
    return w->type == VB_TYPE_F16 && w->K % GM_BK == 0;
}

bool gemm_supported(vb_weight w, int64_t M) {
    if (M < 16 || !encode_fn()) return false;
    if (w->type == VB_TYPE_Q8_0) return w->K % GM_BK == 0;
    if (w->type == VB_TYPE_F16) return w->K % GM_BK == 0;
    return false;
}

int launch_gemm(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, int64_t x_mod,
                const MatmulOut &out, const GemmPro *pro) {
    if (w->type == VB_TYPE_Q8_0 && w->K % GI_BK == 0 &&
        (gemm_small_m(ctx, w, M) || ctx->gemm_i8 == 2 || (ctx->gemm_i8 == 1 && gemm_i8_faster(M, w->K, w->N))))
        return launch_gemm_i8(ctx, w, x, M, ldx, x_mod, out, pro);
    GemmState *gs = gemm_state(ctx);
    if (!gs) return set_error(ctx, VB_ERR_OOM, "gemm: state allocation failed");
    const bool q8 = w->type == VB_TYPE_Q8_0;
    const int K = (int)w->K, N = (int)w->N;
    // Tile width and K split (choices measured on B200).  F16: the widest
    // tile that still gives about one tile per SM, then a K split only when
    // tiles are scarce.  Q8_0 (three MMAs per k-step, so per-unit work is
    // heavier): a small cost model of the persistent grid, time ~ waves x
    // (BN x k-tiles per unit + a fixed per-unit overhead) + the split-K
    // reduction (the last CTA of a tile reads every split's partials in
    // turn: ~40 units per split per 16 columns above M = 128, fitted to
    // M = 1408 sweeps of splits 1-4 x BN 64-128).
    const int tiles_n = (N + GM_BM - 1) / GM_BM;
    const int mr = (int)((M + 15) / 16 * 16);
    const int kt_total = K / GM_BK;
    int BN = 0, splits = 1;
    if (!q8) {
        BN = std::min(256, mr);
        for (int cand : {256, 128, 64}) {
            if (cand > mr) continue;
            BN = cand;
            if ((int64_t)tiles_n * ((M + cand - 1) / cand) * 5 >= (int64_t)ctx->sm_count * 4) break;
        }
        const int64_t tiles0 = (int64_t)tiles_n * ((M + BN - 1) / BN);
        if (tiles0 * 5 < (int64_t)ctx->sm_count * 4)
            splits = (int)std::min<int64_t>(std::max<int64_t>(1, ctx->sm_count / tiles0), std::max(1, kt_total / 2));
    } else {
        double best = 1e300;
        for (int cand : {128, 64, 32, 16}) {
            if (cand > mr && (cand >> 1) >= mr) continue;   // no wider than M needs
            if (cand == 16 && M > 128) continue;             // N = 16 MMAs: issue-bound, measured slower
            const int64_t tiles = (int64_t)tiles_n * ((M + cand - 1) / cand);
            for (int sp = 1; sp <= std::max(1, kt_total / 2); sp++) {
                const int kps = (kt_total + sp - 1) / sp;
                const int64_t units = tiles * ((kt_total + kps - 1) / kps);
                const int64_t waves = (units + ctx->sm_count - 1) / ctx->sm_count;
                // M <= 128 keeps a light split price: its shorter accumulation
                // chains hold the tightest (stage-level) parity gates
                const double split_cost = M > 128 ? 40.0 * sp * (cand / 16) : 0.02 * sp * cand;
                const double t = (double)waves * ((double)cand * kps + 2048.0) + (sp > 1 ? split_cost : 0.0);
                if (t < best * 0.999) { best = t; BN = cand; splits = sp; }
                if (units >= 4 * ctx->sm_count) break;
            }
        }
    }
    if (BN == 0) {      // no candidate passed the filters (not expected): one plain tile width
        BN = std::min(64, mr);
        splits = 1;
    }
    const int tiles_m = (int)((M + BN - 1) / BN);
    const int tiles = tiles_m * tiles_n;
    const int kt_per_split = (kt_total + splits - 1) / splits;
    splits = (kt_total + kt_per_split - 1) / kt_per_split;
    if (tiles > 65536) return set_error(ctx, VB_ERR_INVALID_ARG, "gemm: too many tiles");

    const uint32_t a_bytes = q8 ? GM_BM * GM_BK : GM_BM * GM_BK * 2;
    const uint32_t b_bytes = (uint32_t)BN * 128;
    const uint32_t stage = a_bytes + b_bytes * (q8 ? 2 : 1);
    const int n_conv = q8 ? 2 : 1;
    const size_t conv_bytes = q8 ? (size_t)n_conv * 32768 : 0;
    int n_tma = (int)std::min<size_t>(GM_MAX_STAGES, (GM_SMEM_BUDGET - conv_bytes) / stage);
    if (n_tma < 2) return set_error(ctx, VB_ERR_INVALID_ARG, "gemm: tile does not fit shared memory");
    const size_t smem = (size_t)n_tma * stage + conv_bytes + 1024;
    uint32_t pcols = 32;
    while (pcols < (uint32_t)BN) pcols <<= 1;
    // two accumulator buffers (the epilogue of one tile overlaps the next
    // tile's MMAs); Q8_0 keeps the hi*hi and cross-term sums side by side
    // in each (BN <= 128, so at most 4 x 128 columns)
    const uint32_t cols = (q8 ? 4u : 2u) * pcols;

    // activation operands
    const size_t ab = (size_t)M * K * 2;
    int rc = arena_reserve(ctx, gs->act, 2 * ab + 512);
    if (rc) return rc;
    __half *bh = (__half *)gs->act.ptr;
    __half *bl = (__half *)((uint8_t *)gs->act.ptr + ((ab + 255) & ~(size_t)255));
    {
        const int64_t items = M * (K / 8);
        const int64_t lx = ldx ? ldx : (pro && pro->swiglu_f ? 2 * (int64_t)K : K);
        const int vec = ((uintptr_t)x % 16 == 0) && (lx % 4 == 0);
        const int64_t xm = x_mod > 0 ? x_mod : M;
        if (pro && pro->norm_w) {
            if (K > 8 * ACT_NORM_THREADS * ACT_NORM_ITEMS)
                return set_error(ctx, VB_ERR_INVALID_ARG, "gemm: fused RMSNorm row of %d values is too wide", K);
            VB_CHECK(ctx, pdl_launch(ctx, gemm_act_norm_kernel, dim3((unsigned)M), dim3(ACT_NORM_THREADS), 0, x, lx, xm,
                                     K, q8 ? 1 : 0, ctx->qrule, vec, pro->norm_w, pro->eps, bh, bl));
        } else {
            VB_CHECK(ctx, pdl_launch(ctx, gemm_act_kernel, dim3((unsigned)((items + 255) / 256)), dim3(256), 0, x, lx,
                                     xm, (int)M, K, q8 ? 1 : 0, ctx->qrule, vec, pro ? pro->swiglu_f : 0, bh, bl));
        }
        VB_LAUNCH_CHECK(ctx, "gemm_act");
    }
    // descriptors: the weight's once per weight, the activations' per shape
    if (!w->tmap_ok) {
        CUtensorMap *tw = reinterpret_cast<CUtensorMap *>(w->tmap);
        w->tmap_ok = q8 ? make_map(tw, w->data, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, GM_BK, GM_BM, false)
                        : make_map(tw, w->data, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, N, GM_BK, GM_BM, true);
        if (!w->tmap_ok) return set_error(ctx, VB_ERR_BACKEND, "gemm: weight tensor map encoding failed");
    }
    const void *blp = q8 ? (const void *)bl : (const void *)bh;
    ActMaps *am = nullptr;
    for (ActMaps &c : gs->cache)
        if (c.bh == bh && c.bl == blp && c.K == K && c.M == (int)M && c.BN == BN && !c.tf32 && !c.i8) am = &c;
    if (!am) {
        am = &gs->cache[gs->next];
        gs->next = (gs->next + 1) % 8;
        am->bh = nullptr;
        if (!make_map(&am->th, bh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, M, GM_BK, BN, true) ||
            !make_map(&am->tl, blp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, M, GM_BK, BN, true))
            return set_error(ctx, VB_ERR_BACKEND, "gemm: activation tensor map encoding failed");
        am->bh = bh;
        am->bl = blp;
        am->K = K;
        am->M = (int)M;
        am->BN = BN;
        am->tf32 = false;
        am->i8 = false;
    }

    GemmArgs g{};
    g.q8 = q8;
    g.bk = GM_BK;
    g.K = K;
    g.N = N;
    g.M = (int)M;
    g.BN = BN;
    g.kt_total = kt_total;
    g.kt_per_split = kt_per_split;
    g.splits = splits;
    g.tiles_m = tiles_m;
    g.tiles_n = tiles_n;
    g.n_tma = n_tma;
    g.n_conv = n_conv;
    g.tmem_cols = cols;
    g.small_off = q8 ? pcols : 0u;
    g.sc = w->scales;
    g.y = out.y;
    g.bias = out.bias;
    g.flags = out.flags;
    g.res = out.res;
    g.res_scale = out.res_scale;
    g.ldy = out.ldy ? out.ldy : N;
    g.seg = out.seg ? out.seg : M;
    g.seg_stride = out.seg ? out.seg_stride : 0;
    g.seg_off = out.seg ? out.seg_off : 0;
    g.seg_plain = g.seg >= M && g.seg_off == 0;
    g.cnt = gs->cnt;
    g.err = gs->err;
    if (splits > 1) {
        g.Mp = tiles_m * BN;
        rc = arena_reserve(ctx, gs->part, (size_t)splits * N * g.Mp * 4);
        if (rc) return rc;
        g.ws = (float *)gs->part.ptr;
    }
    const int n_work = tiles * splits;
    const CUtensorMap &twm = *reinterpret_cast<const CUtensorMap *>(w->tmap);
    VB_CHECK(ctx, pdl_launch(ctx, gemm_kernel<false>, dim3((unsigned)std::min(n_work, ctx->sm_count)),
                             dim3(GM_THREADS), smem, twm, twm, am->th, am->tl, g));
    VB_LAUNCH_CHECK(ctx, "gemm");
    return VB_OK;
}

// fp32 GEMM as three tf32 products (the AudioVAE convolutions):
// y[m][n] = sum_k W[n][k] * A[m][k] with both operands given as tf32 hi/lo
// splits (hi = tf32(v), lo = tf32(v - hi), each stored as fp32 with the low
// 13 mantissa bits clear): hi*hi + hi*lo + lo*hi in fp32, so every product
// carries ~22 significant bits, as an fp32 multiply-add's does to within a
// few units of 2^-22.  The AudioVAE epilogue (bias period cb, residual skip,
// sr_cond, Snake) is fused.
int launch_gemm_tf32(vb_ctx *ctx, Tf32Weight &w, const float *a_hi, const float *a_lo, int64_t M,
                     const GemmEpi &e) {
    GemmState *gs = gemm_state(ctx);
    if (!gs) return set_error(ctx, VB_ERR_OOM, "gemm: state allocation failed");
    const int K = w.K, N = w.N, BK = 32;
    if (K % BK || M < 1 || !encode_fn())
        return set_error(ctx, VB_ERR_INVALID_ARG, "gemm_tf32: K must be a multiple of 32");
    if (((uintptr_t)a_hi | (uintptr_t)a_lo) % 16)
        return set_error(ctx, VB_ERR_INVALID_ARG, "gemm_tf32: operands must be 16-byte aligned");
    const int tiles_n = (N + GM_BM - 1) / GM_BM;
    const int mr = (int)((M + 15) / 16 * 16);
    const int kt_total = K / BK;
    // the widest tile that still gives about one tile per SM, a K split
    // when tiles are scarce (as the F16 path)
    // (BN <= 128: each accumulator buffer holds the hi*hi and the cross-term
    // sums side by side, two buffers -> 4 x 128 TMEM columns)
    int BN = std::min(128, mr), splits = 1;
    for (int cand : {128, 64}) {
        if (cand > mr) continue;
        BN = cand;
        if ((int64_t)tiles_n * ((M + cand - 1) / cand) * 5 >= (int64_t)ctx->sm_count * 4) break;
    }
    const int64_t tiles0 = (int64_t)tiles_n * ((M + BN - 1) / BN);
    if (tiles0 * 5 < (int64_t)ctx->sm_count * 4)
        splits = (int)std::min<int64_t>(std::max<int64_t>(1, ctx->sm_count / tiles0), std::max(1, kt_total / 2));
    // at most 1024 k per accumulation: longer sums are finished by the
    // split-K reduction (fp32, round to nearest, split order)
    splits = std::max(splits, (K + 1023) / 1024);
    const int tiles_m = (int)((M + BN - 1) / BN);
    const int tiles = tiles_m * tiles_n;
    const int kt_per_split = (kt_total + splits - 1) / splits;
    splits = (kt_total + kt_per_split - 1) / kt_per_split;
    if (tiles > 65536) return set_error(ctx, VB_ERR_INVALID_ARG, "gemm_tf32: too many tiles");
    const uint32_t stage = 2u * GM_BM * 128 + 2u * (uint32_t)BN * 128;
    const int n_tma = (int)std::min<size_t>(GM_MAX_STAGES, (size_t)GM_SMEM_BUDGET / stage);
    if (n_tma < 2) return set_error(ctx, VB_ERR_INVALID_ARG, "gemm_tf32: tile does not fit shared memory");
    const size_t smem = (size_t)n_tma * stage + 1024;
    uint32_t pcols = 32;
    while (pcols < (uint32_t)BN) pcols <<= 1;
    const uint32_t cols = 4 * pcols;      // 2 buffers x (hi*hi, cross terms)
    if (!w.maps_ok) {
        w.maps_ok = make_map(reinterpret_cast<CUtensorMap *>(w.map_hi), w.hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K, N,
                             BK, GM_BM, true) &&
                    make_map(reinterpret_cast<CUtensorMap *>(w.map_lo), w.lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K, N,
                             BK, GM_BM, true);
        if (!w.maps_ok) return set_error(ctx, VB_ERR_BACKEND, "gemm_tf32: weight tensor map encoding failed");
    }
    ActMaps *am = nullptr;
    for (ActMaps &c : gs->cache)
        if (c.bh == a_hi && c.bl == a_lo && c.K == K && c.M == (int)M && c.BN == BN && c.tf32 && !c.i8) am = &c;
    if (!am) {
        am = &gs->cache[gs->next];
        gs->next = (gs->next + 1) % 8;
        am->bh = nullptr;
        if (!make_map(&am->th, a_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K, M, BK, BN, true) ||
            !make_map(&am->tl, a_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K, M, BK, BN, true))
            return set_error(ctx, VB_ERR_BACKEND, "gemm_tf32: activation tensor map encoding failed");
        am->bh = a_hi;
        am->bl = a_lo;
        am->K = K;
        am->M = (int)M;
        am->BN = BN;
        am->tf32 = true;
        am->i8 = false;
    }
    GemmArgs g{};
    g.bk = BK;
    g.K = K;
    g.N = N;
    g.M = (int)M;
    g.BN = BN;
    g.kt_total = kt_total;
    g.kt_per_split = kt_per_split;
    g.splits = splits;
    g.tiles_m = tiles_m;
    g.tiles_n = tiles_n;
    g.n_tma = n_tma;
    g.n_conv = 1;
    g.tmem_cols = cols;
    g.y = e.y;
    g.bias = e.bias;
    g.ldy = N;
    g.seg = M;
    g.seg_plain = 1;
    g.cnt = gs->cnt;
    g.err = gs->err;
    g.small_off = pcols;
    g.cb = e.cb > 0 ? e.cb : N;
    g.skip = e.skip;
    g.out_x = e.out_x;
    g.alpha = e.alpha;
    g.sr_scale = e.sr_scale;
    g.sr_bias = e.sr_bias;
    if (splits > 1) {
        g.Mp = tiles_m * BN;
        const int rc = arena_reserve(ctx, gs->part, (size_t)splits * N * g.Mp * 4);
        if (rc) return rc;
        g.ws = (float *)gs->part.ptr;
    }
    const int n_work = tiles * splits;
    gemm_kernel<true><<<(unsigned)std::min(n_work, ctx->sm_count), GM_THREADS, smem, ctx->stream>>>(
        *reinterpret_cast<const CUtensorMap *>(w.map_hi), *reinterpret_cast<const CUtensorMap *>(w.map_lo), am->th,
        am->tl, g);
    VB_LAUNCH_CHECK(ctx, "gemm_tf32");
    return VB_OK;
}

int *gemm_error_word(vb_ctx *ctx) {
    GemmState *gs = gemm_state(ctx);
    return gs ? gs->err : nullptr;
}

int gemm_device_error(vb_ctx *ctx, int *code) {
    GemmState *gs = static_cast<GemmState *>(ctx->gemm);
    *code = 0;
    if (!gs) return VB_OK;
    VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
    VB_CHECK(ctx, cudaMemcpy(code, gs->err, sizeof(int), cudaMemcpyDeviceToHost));
    return VB_OK;
}

}  // namespace vb
