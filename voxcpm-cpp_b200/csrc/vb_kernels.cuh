// vb_kernels.cuh -- launchers shared between the translation units.
#pragma once

#include "vb_common.cuh"

namespace vb {

int init_kernels(vb_ctx *ctx);

// weights (vb_quant.cu)
int weight_upload(vb_ctx *ctx, int type, int64_t K, int64_t N, const void *host, size_t nbytes, vb_weight *out);
void weight_free(vb_ctx *ctx, vb_weight w);
// A new F32 weight [out_dim][in_dim] holding element j*out_dim + o of the
// flat storage of src at row o, column j (src keeps its own storage).
int weight_transpose_f32(vb_ctx *ctx, vb_weight src, int64_t in_dim, int64_t out_dim, vb_weight *out);

// Output mapping of a mat-mul: logical row m of the [M][N] result lands in
// row  (m / seg) * seg_stride + seg_off + (m % seg)  of y (leading dim ldy).
// With seg = M, seg_stride = 0, seg_off = 0, ldy = N it is the plain layout.
struct MatmulOut {
    float *y = nullptr;
    const float *bias = nullptr;   // [N] or null
    unsigned flags = 0;            // VB_OUT_BF16
    int64_t ldy = 0;
    int64_t seg = 0, seg_stride = 0, seg_off = 0;
    // residual epilogue: y = bf16(res + res_scale * value), value after bias
    // and the bf16 flag (block residual, src/minicpm4.c:496-528); res rows
    // follow y's mapping and may alias y
    const float *res = nullptr;
    float res_scale = 1.0f;
};

// Input mapping: logical row m reads x row (m % x_mod) (x_mod = M: plain),
// leading dimension ldx.
int launch_matmul(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, int64_t x_mod,
                  const MatmulOut &out);

// Tensor-core path for M >= 16 (vb_gemm.cu); launch_matmul dispatches to it.
bool gemm_supported(vb_weight w, int64_t M);
bool gemm_small_m(const vb_ctx *ctx, vb_weight w, int64_t M);
// Prologue fused into the tensor-core path's activation operand: norm_w set
// -> the operand is vcpm_rms_norm(x) with weight norm_w and bf16 rounding;
// swiglu_f > 0 -> x rows are [gate (F) | up (F)] (ldx 0 means 2F) and the
// operand is the SwiGLU middle of vcpm_mlp.
struct GemmPro {
    const float *norm_w = nullptr;
    float eps = 0.0f;
    int swiglu_f = 0;
};
int launch_gemm(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, int64_t x_mod,
                const MatmulOut &out, const GemmPro *pro = nullptr);
// True when launch_matmul takes the tensor-core path for this weight and M
// (so a GemmPro prologue can be fused).
bool matmul_uses_gemm(vb_ctx *ctx, vb_weight w, int64_t M);
// launch_matmul through the tensor-core path with a fused prologue; the
// caller checks matmul_uses_gemm first.
int launch_matmul_pro(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, const GemmPro &pro,
                      const MatmulOut &out);
int gemm_device_error(vb_ctx *ctx, int *code);
// The context's device error word of the mat-mul kernels (created on first
// use): a bounded wait that runs out records its code there.
int *gemm_error_word(vb_ctx *ctx);
// vb_matmul for M <= 8 on a Q8_0 / F16 weight through the weight-streaming
// kernel as a single op (vb_stream.cu); -1 when the shape is not supported
// there (the caller then takes the per-launch GEMV kernel).
int launch_stream1(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, int64_t x_mod,
                   const MatmulOut &out);
void gemm_free(vb_ctx *ctx);

int launch_quantize_q8_0(vb_ctx *ctx, const float *x, int64_t K, int64_t M, void *blocks, int rule);
int launch_dequantize_q8_0(vb_ctx *ctx, const void *blocks, int64_t n, float *y);
int launch_get_rows(vb_ctx *ctx, vb_weight w, const int32_t *ids, int64_t n, float *y);

// fp32 GEMM through three tf32 tensor-core products (vb_gemm.cu).  Weights
// [N][K] pre-split into tf32 hi/lo (fp32 storage, low 13 mantissa bits
// clear); the TMA descriptors are encoded on first use.
struct Tf32Weight {
    float *hi = nullptr, *lo = nullptr;
    int K = 0, N = 0;
    alignas(64) unsigned char map_hi[128];
    alignas(64) unsigned char map_lo[128];
    bool maps_ok = false;
};
// AudioVAE epilogue: v = acc + bias[n % cb] (+ skip[m][n]); y[m][n] = v
// (if y); out_x[m][n] = snake(alpha)(v * sr_scale + sr_bias) (if out_x).
struct GemmEpi {
    float *y = nullptr;
    const float *bias = nullptr;
    int cb = 0;
    const float *skip = nullptr;
    float *out_x = nullptr;
    const float *alpha = nullptr, *sr_scale = nullptr, *sr_bias = nullptr;
};
int launch_gemm_tf32(vb_ctx *ctx, Tf32Weight &w, const float *a_hi, const float *a_lo, int64_t M, const GemmEpi &e);

// elementwise (vb_elem.cu)
int launch_rms_norm(vb_ctx *ctx, const float *x, const float *w, float *y, int64_t n, int64_t rows, float eps,
                    unsigned flags, int64_t ldx = 0, int64_t ldy = 0);
int launch_bf16_round(vb_ctx *ctx, float *x, int64_t n);
int launch_residual(vb_ctx *ctx, const float *a, const float *b, float scale, float *y, int64_t n, unsigned flags);
int launch_swiglu(vb_ctx *ctx, const float *g, const float *u, float *y, int64_t n, unsigned flags);
int launch_fsq(vb_ctx *ctx, float *x, int64_t n, float s);
// In-place NEOX rotation of x (row t at x + t*ldx, n_heads x head_dim),
// positions pos[t]; table cs [max_pos][head_dim].
int launch_rope(vb_ctx *ctx, float *x, int64_t ldx, int head_dim, int n_heads, int T, const int32_t *pos,
                const float *cs, unsigned flags);
// RoPE of q and k (bf16) and the bf16 K/V append in one launch; kd = the
// k block's width (v starts kd after k in a row).
int launch_rope_kv(vb_ctx *ctx, float *qkv, int64_t ld, int64_t kd, int head_dim, int n_heads, int n_kv, int T,
                   const int32_t *pos, const float *cs, uint16_t *kc, uint16_t *vc, int n_rows, const int32_t *dst_row);
int launch_kv_write(vb_ctx *ctx, const float *k, const float *v, int64_t ldkv, uint16_t *kc, uint16_t *vc,
                    int n_rows, int T, int n_kv, int head_dim, const int32_t *dst_row);
int launch_fill(vb_ctx *ctx, float *x, float v, int64_t n);

// attention (vb_attn.cu)
// Bidirectional attention over n_seg uniform segments of T <= 32 tokens
// (token t of segment s attends to K/V rows s*T .. s*T+T-1): one CTA per
// (segment, KV group) stages the segment's K/V once for all its tokens.
int launch_attention_segments(vb_ctx *ctx, const float *q, int64_t ldq, const uint16_t *k, const uint16_t *v,
                              int n_rows, int n_seg, int T, int n_heads, int n_kv, int head_dim, float *out,
                              int64_t ldo);
int launch_attention(vb_ctx *ctx, const float *q, int64_t ldq, const uint16_t *k, const uint16_t *v, int n_rows,
                     int T, int n_heads, int n_kv, int head_dim, const int32_t *row_start, const int32_t *kv_len,
                     int max_kv_len, float *out, int64_t ldo);
size_t attention_scratch_bytes(int T, int n_heads, int head_dim, int max_kv_len);

}  // namespace vb
