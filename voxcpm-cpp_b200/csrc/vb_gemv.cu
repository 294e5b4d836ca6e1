// vb_gemv.cu -- ggml_mul_mat on Q8_0 / F16 / F32 weights for small M
// (decode GEMV and the small-batch case).
//
// Semantics (ggml-CPU, the parity target): for a Q8_0 weight every
// activation row is first quantized to Q8_0 and each output is
//     y[m][n] = sum_b  float(isum_b) * (d_w[n][b] * d_x[m][b])
// with isum_b the exact int32 dot of the 32 int8 pairs of block b; for F16 the
// activation is rounded to fp16 and products accumulate in fp32.
//
// Mapping: 256-thread CTAs, each warp owns RPW weight rows.  A CTA first
// converts up to MC activation rows into shared memory (Q8_0: int8 values +
// fp32 copies of the fp16 scales, exactly the values the oracle uses), then
// every lane streams 16-byte chunks of its rows with non-allocating vector
// loads (U chunks in flight per row) and does 4 dp4a per chunk and row.
// Partial sums are combined with a warp shuffle tree; lane 0 applies the
// epilogue (bias, bf16 rounding, strided/segmented output rows).
// The kernel is bound by HBM: 34/32 bytes per weight, each read once.
#include "vb_common.cuh"
#include "vb_kernels.cuh"
#include "vb_device.cuh"

namespace vb {

struct GemvArgs {
    const void *w;           // qs int8 / fp16 / fp32, [N][K]
    const uint16_t *sc;      // Q8_0 scales [N][K/32]
    int64_t K, N;
    const float *x;
    int64_t M, ldx, x_mod;
    MatmulOut out;
    int rule;
};

__device__ __forceinline__ void gemv_store(const MatmulOut &o, int64_t m, int64_t n, float v) {
    if (o.bias) v = __fadd_rn(v, o.bias[n]);
    if (o.flags & VB_OUT_BF16) v = bf16r(v);
    int64_t row = (m / o.seg) * o.seg_stride + o.seg_off + (m % o.seg);
    if (o.res) {
        if (o.res_scale != 1.0f) v = __fmul_rn(v, o.res_scale);
        v = bf16r(__fadd_rn(o.res[row * o.ldy + n], v));
    }
    o.y[row * o.ldy + n] = v;
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// ----------------------------------------------------------------- Q8_0
template <int MC, int RPW, int U>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_q8_kernel(GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int64_t K = a.K, N = a.N, nb = K / QK, nch = K / 16;
    int8_t *sq = reinterpret_cast<int8_t *>(smem);                       // [MC][K]
    float *sd = reinterpret_cast<float *>(smem + ((MC * K + 15) & ~15));  // [MC][nb]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = ((int64_t)blockIdx.x * GEMV_WARPS + warp) * RPW;
    const int8_t *qs = reinterpret_cast<const int8_t *>(a.w);

    for (int64_t m0 = 0; m0 < a.M; m0 += MC) {
        const int mc = (int)((a.M - m0) < MC ? (a.M - m0) : MC);
        __syncthreads();
        for (int64_t blk = warp; blk < (int64_t)mc * nb; blk += GEMV_WARPS) {
            const int64_t m = blk / nb, b = blk % nb;
            const int64_t xr = (m0 + m) % a.x_mod;
            float v = a.x[xr * a.ldx + b * QK + lane];
            int q;
            uint16_t dh;
            q8_quant_warp(v, a.rule, q, dh);
            sq[m * K + b * QK + lane] = (int8_t)q;
            if (lane == 0) sd[m * nb + b] = h2f(dh);
        }
        __syncthreads();

        float acc[RPW][MC];
#pragma unroll
        for (int r = 0; r < RPW; r++)
#pragma unroll
            for (int m = 0; m < MC; m++) acc[r][m] = 0.0f;

        for (int64_t c0 = lane; c0 < nch; c0 += 32 * U) {
            int4 wv[U][RPW];
            float sw[U][RPW];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t c = c0 + 32 * u;
#pragma unroll
                for (int r = 0; r < RPW; r++) {
                    const int64_t row = row0 + r;
                    if (c < nch && row < N) {
                        wv[u][r] = ldg_stream(qs + row * K + c * 16);
                        sw[u][r] = h2f(__ldg(a.sc + row * nb + (c >> 1)));
                    } else {
                        wv[u][r] = make_int4(0, 0, 0, 0);
                        sw[u][r] = 0.0f;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t c = c0 + 32 * u;
                if (c < nch) {
#pragma unroll
                    for (int m = 0; m < MC; m++) {
                        if (m < mc) {
                            const int4 xv = *reinterpret_cast<const int4 *>(sq + m * K + c * 16);
                            const float dx = sd[m * nb + (c >> 1)];
#pragma unroll
                            for (int r = 0; r < RPW; r++) {
                                const int s = dot16_i8(wv[u][r], xv);
                                acc[r][m] = fmaf((float)s, __fmul_rn(sw[u][r], dx), acc[r][m]);
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RPW; r++)
#pragma unroll
            for (int m = 0; m < MC; m++) {
                if (m < mc) {
                    float v = warp_sum(acc[r][m]);
                    if (lane == 0 && row0 + r < N) gemv_store(a.out, m0 + m, row0 + r, v);
                }
            }
    }
}

// -------------------------------------------------------------- F16 / F32
template <int MC, int RPW, int U, bool F16>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_fp_kernel(GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int EB = F16 ? 2 : 4;          // element bytes
    constexpr int EPC = 16 / EB;             // elements per 16-byte chunk
    const int64_t K = a.K, N = a.N, nch = K / EPC;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = ((int64_t)blockIdx.x * GEMV_WARPS + warp) * RPW;
    const uint8_t *wb = reinterpret_cast<const uint8_t *>(a.w);

    for (int64_t m0 = 0; m0 < a.M; m0 += MC) {
        const int mc = (int)((a.M - m0) < MC ? (a.M - m0) : MC);
        __syncthreads();
        for (int64_t i = threadIdx.x; i < (int64_t)mc * K; i += GEMV_THREADS) {
            const int64_t m = i / K, k = i % K;
            const float v = a.x[((m0 + m) % a.x_mod) * a.ldx + k];
            if (F16) reinterpret_cast<uint16_t *>(smem)[m * K + k] = f2h(v);
            else reinterpret_cast<float *>(smem)[m * K + k] = v;
        }
        __syncthreads();

        float acc[RPW][MC];
#pragma unroll
        for (int r = 0; r < RPW; r++)
#pragma unroll
            for (int m = 0; m < MC; m++) acc[r][m] = 0.0f;

        for (int64_t c0 = lane; c0 < nch; c0 += 32 * U) {
            int4 wv[U][RPW];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t c = c0 + 32 * u;
#pragma unroll
                for (int r = 0; r < RPW; r++) {
                    const int64_t row = row0 + r;
                    wv[u][r] = (c < nch && row < N) ? ldg_stream(wb + (row * K + c * EPC) * EB)
                                                    : make_int4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t c = c0 + 32 * u;
                if (c < nch) {
#pragma unroll
                    for (int m = 0; m < MC; m++) {
                        if (m < mc) {
                            // one 16-byte register copy of the activation piece, shared by the rows
                            // (a reference into shared memory would be re-read as 4-byte loads)
                            const int4 xv = *reinterpret_cast<const int4 *>(smem + (m * K + c * EPC) * EB);
#pragma unroll
                            for (int r = 0; r < RPW; r++) {
                                if (F16) acc[r][m] = dot8_f16(wv[u][r], xv, acc[r][m]);
                                else acc[r][m] = dot4_f32(wv[u][r], make_float4(__int_as_float(xv.x), __int_as_float(xv.y),
                                                                                 __int_as_float(xv.z), __int_as_float(xv.w)),
                                                          acc[r][m]);
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RPW; r++)
#pragma unroll
            for (int m = 0; m < MC; m++) {
                if (m < mc) {
                    float v = warp_sum(acc[r][m]);
                    if (lane == 0 && row0 + r < N) gemv_store(a.out, m0 + m, row0 + r, v);
                }
            }
    }
}

// Scalar fallback for shapes the vector kernels cannot take (K not a
// multiple of the 16-byte chunk, e.g. the 4- and 8-wide unit fixtures):
// one warp per (m, n) output.
__global__ void gemv_scalar_kernel(GemvArgs a, int type) {
    const int64_t o = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (o >= a.M * a.N) return;
    const int64_t m = o / a.N, n = o % a.N;
    const float *x = a.x + (m % a.x_mod) * a.ldx;
    float acc = 0.0f;
    if (type == VB_TYPE_Q8_0) {
        const int8_t *qs = reinterpret_cast<const int8_t *>(a.w) + n * a.K;
        const int64_t nb = a.K / QK;
        for (int64_t b = 0; b < nb; b++) {
            int q;
            uint16_t dh;
            q8_quant_warp(x[b * QK + lane], a.rule, q, dh);
            int s = q * (int)qs[b * QK + lane];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            acc = fmaf((float)s, __fmul_rn(h2f(a.sc[n * nb + b]), h2f(dh)), acc);
        }
    } else {
        float part = 0.0f;
        for (int64_t k = lane; k < a.K; k += 32) {
            float wv, xv = x[k];
            if (type == VB_TYPE_F16) {
                wv = h2f(reinterpret_cast<const uint16_t *>(a.w)[n * a.K + k]);
                xv = h2f(f2h(xv));
            } else {
                wv = reinterpret_cast<const float *>(a.w)[n * a.K + k];
            }
            part = fmaf(wv, xv, part);
        }
        acc = warp_sum(part);
    }
    if (lane == 0) gemv_store(a.out, m, n, acc);
}

// ------------------------------------------------------------------ launch
template <typename KernelT>
static int set_smem(vb_ctx *ctx, KernelT k, size_t bytes) {
    VB_CHECK(ctx, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return VB_OK;
}

constexpr size_t GEMV_SMEM_MAX = 96 * 1024;

int init_gemv(vb_ctx *ctx) {
    int rc = 0;
    rc |= set_smem(ctx, gemv_q8_kernel<1, 2, 4>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_q8_kernel<2, 2, 4>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_q8_kernel<4, 2, 2>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_q8_kernel<8, 2, 2>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<1, 2, 4, true>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<2, 2, 4, true>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<4, 2, 2, true>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<8, 2, 2, true>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<1, 2, 4, false>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<2, 2, 4, false>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<4, 2, 2, false>, GEMV_SMEM_MAX);
    rc |= set_smem(ctx, gemv_fp_kernel<8, 2, 2, false>, GEMV_SMEM_MAX);
    return rc ? VB_ERR_BACKEND : VB_OK;
}

static size_t q8_smem(int mc, int64_t K) { return (size_t)((mc * K + 15) & ~15) + (size_t)mc * (K / QK) * 4; }

bool matmul_uses_gemm(vb_ctx *ctx, vb_weight w, int64_t M) {
    return ctx->use_gemm && (gemm_supported(w, M) || gemm_small_m(ctx, w, M));
}

int launch_matmul_pro(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, const GemmPro &pro,
                      const MatmulOut &out_in) {
    if (!w || !x || !out_in.y || M < 0) return set_error(ctx, VB_ERR_INVALID_ARG, "matmul: bad argument");
    if (M == 0) return VB_OK;
    if (!matmul_uses_gemm(ctx, w, M)) return set_error(ctx, VB_ERR_INVALID_ARG, "matmul: fused prologue needs M >= 16");
    MatmulOut out = out_in;
    if (out.ldy == 0) out.ldy = w->N;
    if (out.seg == 0) { out.seg = M; out.seg_stride = 0; out.seg_off = 0; }
    return launch_gemm(ctx, w, x, M, ldx, 0, out, &pro);
}

int launch_matmul(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, int64_t x_mod,
                  const MatmulOut &out_in) {
    if (!w || !x || !out_in.y || M < 0) return set_error(ctx, VB_ERR_INVALID_ARG, "matmul: bad argument");
    if (M == 0) return VB_OK;
    MatmulOut out = out_in;
    if (out.ldy == 0) out.ldy = w->N;
    if (out.seg == 0) { out.seg = M; out.seg_stride = 0; out.seg_off = 0; }
    if (matmul_uses_gemm(ctx, w, M)) return launch_gemm(ctx, w, x, M, ldx, x_mod, out);
    {
        // small M on Q8_0 / F16: the weight-streaming kernel as a single op
        const int rc = launch_stream1(ctx, w, x, M, ldx ? ldx : w->K, x_mod > 0 ? x_mod : M, out);
        if (rc >= 0) return rc;
    }
    GemvArgs a;
    a.w = w->data;
    a.sc = w->scales;
    a.K = w->K;
    a.N = w->N;
    a.x = x;
    a.M = M;
    a.ldx = ldx ? ldx : w->K;
    a.x_mod = x_mod > 0 ? x_mod : M;
    a.out = out;
    a.rule = ctx->qrule;
    const int64_t K = w->K;
    const int rows_per_cta = GEMV_WARPS * 2;
    const unsigned grid = (unsigned)((w->N + rows_per_cta - 1) / rows_per_cta);

    if (w->type == VB_TYPE_Q8_0) {
        int mc = M >= 8 ? 8 : (M >= 4 ? 4 : (M >= 2 ? 2 : 1));
        while (mc > 1 && q8_smem(mc, K) > GEMV_SMEM_MAX) mc >>= 1;
        if (q8_smem(mc, K) > GEMV_SMEM_MAX || K % 16) goto scalar;
        size_t sm = q8_smem(mc, K);
        switch (mc) {
            case 1: gemv_q8_kernel<1, 2, 4><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
            case 2: gemv_q8_kernel<2, 2, 4><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
            case 4: gemv_q8_kernel<4, 2, 2><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
            default: gemv_q8_kernel<8, 2, 2><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
        }
        VB_LAUNCH_CHECK(ctx, "gemv_q8");
        return VB_OK;
    } else {
        const bool f16 = w->type == VB_TYPE_F16;
        const int eb = f16 ? 2 : 4;
        if (K % (16 / eb)) goto scalar;
        int mc = M >= 8 ? 8 : (M >= 4 ? 4 : (M >= 2 ? 2 : 1));
        while (mc > 1 && (size_t)mc * K * eb > GEMV_SMEM_MAX) mc >>= 1;
        size_t sm = (size_t)mc * K * eb;
        if (sm > GEMV_SMEM_MAX) goto scalar;
        if (f16) {
            switch (mc) {
                case 1: gemv_fp_kernel<1, 2, 4, true><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
                case 2: gemv_fp_kernel<2, 2, 4, true><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
                case 4: gemv_fp_kernel<4, 2, 2, true><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
                default: gemv_fp_kernel<8, 2, 2, true><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
            }
        } else {
            switch (mc) {
                case 1: gemv_fp_kernel<1, 2, 4, false><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
                case 2: gemv_fp_kernel<2, 2, 4, false><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
                case 4: gemv_fp_kernel<4, 2, 2, false><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
                default: gemv_fp_kernel<8, 2, 2, false><<<grid, GEMV_THREADS, sm, ctx->stream>>>(a); break;
            }
        }
        VB_LAUNCH_CHECK(ctx, "gemv_fp");
        return VB_OK;
    }
scalar : {
    if (w->type == VB_TYPE_Q8_0 && K % QK) return set_error(ctx, VB_ERR_INVALID_ARG, "Q8_0 K not a multiple of 32");
    int64_t outs = M * w->N;
    gemv_scalar_kernel<<<(unsigned)((outs + 7) / 8), 256, 0, ctx->stream>>>(a, w->type);
    VB_LAUNCH_CHECK(ctx, "gemv_scalar");
    return VB_OK;
}
}

}  // namespace vb
