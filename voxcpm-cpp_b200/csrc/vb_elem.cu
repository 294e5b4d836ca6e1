// vb_elem.cu -- the elementwise glue between the mat-muls: RMSNorm, bf16
// casts, residual adds, SwiGLU, FSQ, NEOX RoPE and the bf16 KV append.
//
// Every fp32 operation is written with an explicitly rounded intrinsic
// (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn) so nvcc cannot contract it
// into an FMA: these ops then produce the same bits as the CPU oracle,
// except where a transcendental (expf, tanhf) is involved.
#include "vb_common.cuh"
#include "vb_kernels.cuh"

namespace vb {

// ggml_rms_norm: sum of fp32 squares in double, mean narrowed to fp32,
// scale = 1/sqrtf(mean+eps), y = x*scale; with w: vcpm_rms_norm's
// bf16(bf16(y)*w) (src/minicpm4.c:132-152).  One CTA per row.
__global__ void rms_norm_kernel(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ y,
                                int64_t n, float eps, unsigned flags, int64_t ldx, int64_t ldy) {
    const float *xr = x + (int64_t)blockIdx.x * ldx;
    float *yr = y + (int64_t)blockIdx.x * ldy;
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = xr[i];
        s += (double)__fmul_rn(v, v);
    }
    __shared__ double red[32];
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
        t = warp_sum_d(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float mean = __double2float_rn(__ddiv_rn(red[0], (double)n));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    const bool b16 = flags & VB_OUT_BF16;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        float v = __fmul_rn(xr[i], scale);
        if (b16) v = bf16r(v);
        if (w) {
            v = __fmul_rn(v, w[i]);
            if (b16) v = bf16r(v);
        }
        yr[i] = v;
    }
}

int launch_rms_norm(vb_ctx *ctx, const float *x, const float *w, float *y, int64_t n, int64_t rows, float eps,
                    unsigned flags, int64_t ldx, int64_t ldy) {
    if (rows == 0) return VB_OK;
    if (!x || !y || n <= 0) return set_error(ctx, VB_ERR_INVALID_ARG, "rms_norm: bad argument");
    int threads = n >= 1024 ? 512 : (n >= 256 ? 256 : 64);
    rms_norm_kernel<<<(unsigned)rows, threads, 0, ctx->stream>>>(x, w, y, n, eps, flags, ldx ? ldx : n,
                                                                  ldy ? ldy : n);
    VB_LAUNCH_CHECK(ctx, "rms_norm");
    return VB_OK;
}

__global__ void bf16_round_kernel(float *x, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = bf16r(x[i]);
}

int launch_bf16_round(vb_ctx *ctx, float *x, int64_t n) {
    if (n == 0) return VB_OK;
    bf16_round_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(x, n);
    VB_LAUNCH_CHECK(ctx, "bf16_round");
    return VB_OK;
}

// y = bf16(a + scale*b); scale == 1 adds b directly (src/minicpm4.c:496-505).
__global__ void residual_kernel(const float *a, const float *b, float scale, float *y, int64_t n, unsigned flags) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float s = (scale != 1.0f) ? __fmul_rn(b[i], scale) : b[i];
    float v = __fadd_rn(a[i], s);
    y[i] = (flags & VB_OUT_BF16) ? bf16r(v) : v;
}

int launch_residual(vb_ctx *ctx, const float *a, const float *b, float scale, float *y, int64_t n, unsigned flags) {
    if (n == 0) return VB_OK;
    residual_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(a, b, scale, y, n, flags);
    VB_LAUNCH_CHECK(ctx, "residual");
    return VB_OK;
}

// vcpm_mlp middle: bf16(bf16(silu(bf16(g))) * bf16(u)) (src/minicpm4.c:441-456);
// the up projection is already bf16-rounded by its mat-mul epilogue in the
// model path, rounding it again is the identity.
__global__ void swiglu_kernel(const float *g, const float *u, float *y, int64_t n, unsigned flags) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const bool b16 = flags & VB_OUT_BF16;
    float gv = g[i], uv = u[i];
    if (b16) { gv = bf16r(gv); uv = bf16r(uv); }
    float s = silu_f(gv);
    if (b16) s = bf16r(s);
    float v = __fmul_rn(s, uv);
    y[i] = b16 ? bf16r(v) : v;
}

int launch_swiglu(vb_ctx *ctx, const float *g, const float *u, float *y, int64_t n, unsigned flags) {
    if (n == 0) return VB_OK;
    swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(g, u, y, n, flags);
    VB_LAUNCH_CHECK(ctx, "swiglu");
    return VB_OK;
}

// vcpm_fsq_quantize (src/fsq.c:16-29).
__global__ void fsq_kernel(float *x, int64_t n, float s, float inv) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fmul_rn(roundf(__fmul_rn(tanhf(x[i]), s)), inv);
}

int launch_fsq(vb_ctx *ctx, float *x, int64_t n, float s) {
    if (n == 0 || s <= 0.0f) return VB_OK;
    const float inv = 1.0f / s;
    fsq_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(x, n, s, inv);
    VB_LAUNCH_CHECK(ctx, "fsq");
    return VB_OK;
}

// NEOX rotation (pair i couples element i with i + head_dim/2) from the
// host-built cos/sin table; one thread per pair.
__global__ void rope_kernel(float *x, int64_t ldx, int head_dim, int n_heads, int T, const int32_t *pos,
                            const float *cs, unsigned flags) {
    const int half = head_dim >> 1;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)T * n_heads * half;
    if (i >= total) return;
    const int p = (int)(i % half);
    const int h = (int)((i / half) % n_heads);
    const int t = (int)(i / ((int64_t)half * n_heads));
    float *v = x + (int64_t)t * ldx + (int64_t)h * head_dim;
    const float *c = cs + (int64_t)pos[t] * head_dim + 2 * p;
    const float cv = c[0], sv = c[1];
    const float x0 = v[p], x1 = v[p + half];
    float r0 = __fsub_rn(__fmul_rn(x0, cv), __fmul_rn(x1, sv));
    float r1 = __fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, cv));
    if (flags & VB_OUT_BF16) { r0 = bf16r(r0); r1 = bf16r(r1); }
    v[p] = r0;
    v[p + half] = r1;
}

int launch_rope(vb_ctx *ctx, float *x, int64_t ldx, int head_dim, int n_heads, int T, const int32_t *pos,
                const float *cs, unsigned flags) {
    int64_t total = (int64_t)T * n_heads * (head_dim / 2);
    if (total == 0) return VB_OK;
    rope_kernel<<<(unsigned)((total + 255) / 256), 256, 0, ctx->stream>>>(x, ldx, head_dim, n_heads, T, pos, cs,
                                                                          flags);
    VB_LAUNCH_CHECK(ctx, "rope");
    return VB_OK;
}

// K/V append as bf16: row dst_row[t] of [n_kv][n_rows][head_dim] stores.
__global__ void kv_write_kernel(const float *k, const float *v, int64_t ldkv, uint16_t *kc, uint16_t *vc,
                                int n_rows, int T, int n_kv, int head_dim, const int32_t *dst_row) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)T * n_kv * head_dim;
    if (i >= total) return;
    const int d = (int)(i % head_dim);
    const int g = (int)((i / head_dim) % n_kv);
    const int t = (int)(i / ((int64_t)head_dim * n_kv));
    const int64_t src = (int64_t)t * ldkv + (int64_t)g * head_dim + d;
    const int64_t dst = ((int64_t)g * n_rows + dst_row[t]) * head_dim + d;
    kc[dst] = bf16_bits(k[src]);
    vc[dst] = bf16_bits(v[src]);
}

int launch_kv_write(vb_ctx *ctx, const float *k, const float *v, int64_t ldkv, uint16_t *kc, uint16_t *vc,
                    int n_rows, int T, int n_kv, int head_dim, const int32_t *dst_row) {
    int64_t total = (int64_t)T * n_kv * head_dim;
    if (total == 0) return VB_OK;
    kv_write_kernel<<<(unsigned)((total + 255) / 256), 256, 0, ctx->stream>>>(k, v, ldkv, kc, vc, n_rows, T, n_kv,
                                                                              head_dim, dst_row);
    VB_LAUNCH_CHECK(ctx, "kv_write");
    return VB_OK;
}

// RoPE of the q and k heads of a fused qkv row and the bf16 K/V append, as
// one launch: item (t, head, pair p) of the n_heads query heads rotates
// the pair in place; of the n_kv key heads it rotates the pair in place and
// stores it with the matching value pair into the caches.  The same
// rounding as rope_kernel followed by kv_write_kernel (bf16 rotated values,
// then their bf16 bits).
__global__ void rope_kv_kernel(float *qkv, int64_t ld, int64_t kd, int head_dim, int n_heads, int n_kv, int T,
                               const int32_t *pos, const float *cs, uint16_t *kc, uint16_t *vc, int n_rows,
                               const int32_t *dst_row) {
    const int half = head_dim >> 1;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)T * (n_heads + n_kv) * half;
    if (i >= total) return;
    const int p = (int)(i % half);
    const int hh = (int)((i / half) % (n_heads + n_kv));
    const int t = (int)(i / ((int64_t)half * (n_heads + n_kv)));
    float *row = qkv + (int64_t)t * ld;
    float *v = row + (int64_t)hh * head_dim;   // q heads, then k heads (k follows q in the row)
    const float *c = cs + (int64_t)pos[t] * head_dim + 2 * p;
    const float cv = c[0], sv = c[1];
    const float x0 = v[p], x1 = v[p + half];
    const float r0 = bf16r(__fsub_rn(__fmul_rn(x0, cv), __fmul_rn(x1, sv)));
    const float r1 = bf16r(__fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, cv)));
    v[p] = r0;
    v[p + half] = r1;
    if (hh < n_heads) return;
    const int g = hh - n_heads;
    const float *vv = row + (int64_t)n_heads * head_dim + kd + (int64_t)g * head_dim;
    const int64_t dst = ((int64_t)g * n_rows + dst_row[t]) * head_dim;
    kc[dst + p] = bf16_bits(r0);
    kc[dst + p + half] = bf16_bits(r1);
    vc[dst + p] = bf16_bits(vv[p]);
    vc[dst + p + half] = bf16_bits(vv[p + half]);
}

int launch_rope_kv(vb_ctx *ctx, float *qkv, int64_t ld, int64_t kd, int head_dim, int n_heads, int n_kv, int T,
                   const int32_t *pos, const float *cs, uint16_t *kc, uint16_t *vc, int n_rows, const int32_t *dst_row) {
    const int64_t total = (int64_t)T * (n_heads + n_kv) * (head_dim / 2);
    if (total == 0) return VB_OK;
    rope_kv_kernel<<<(unsigned)((total + 255) / 256), 256, 0, ctx->stream>>>(qkv, ld, kd, head_dim, n_heads, n_kv, T,
                                                                             pos, cs, kc, vc, n_rows, dst_row);
    VB_LAUNCH_CHECK(ctx, "rope_kv");
    return VB_OK;
}

__global__ void fill_kernel(float *x, float v, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = v;
}

int launch_fill(vb_ctx *ctx, float *x, float v, int64_t n) {
    if (n == 0) return VB_OK;
    fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(x, v, n);
    VB_LAUNCH_CHECK(ctx, "fill");
    return VB_OK;
}

}  // namespace vb
