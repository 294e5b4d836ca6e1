// vb_ops.cu -- op-level entry points of the C ABI (include/vcpm_b200.h).
// Each validates its arguments, enqueues on the context stream and returns a
// vcpm_status code; failures leave a message in vb_last_error().
#include "vb_common.cuh"
#include "vb_kernels.cuh"

namespace vb {
int init_gemv(vb_ctx *ctx);
int init_attention(vb_ctx *ctx);
int init_model_kernels(vb_ctx *ctx);
int init_stream(vb_ctx *ctx);
int init_gemm(vb_ctx *ctx);

int init_kernels(vb_ctx *ctx) {
    if (init_gemv(ctx)) return VB_ERR_BACKEND;
    if (init_stream(ctx)) return VB_ERR_BACKEND;
    if (init_attention(ctx)) return VB_ERR_BACKEND;
    if (init_model_kernels(ctx)) return VB_ERR_BACKEND;
    if (init_gemm(ctx)) return VB_ERR_BACKEND;
    return VB_OK;
}
}  // namespace vb

using namespace vb;

#define VB_REQUIRE(ctx, cond, msg)                                          \
    do {                                                                    \
        if (!(ctx)) return VB_ERR_INVALID_ARG;                              \
        if (!(cond)) return vb::set_error((ctx), VB_ERR_INVALID_ARG, "%s", (msg)); \
    } while (0)

extern "C" int vb_matmul(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, float *y, unsigned flags) {
    return vb_matmul_bias(ctx, w, x, M, nullptr, y, flags);
}

extern "C" int vb_matmul_bias(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, const float *bias, float *y,
                              unsigned flags) {
    VB_REQUIRE(ctx, w && x && y && M >= 0, "vb_matmul: null pointer or negative M");
    MatmulOut o;
    o.y = y;
    o.bias = bias;
    o.flags = flags;
    return launch_matmul(ctx, w, x, M, 0, 0, o);
}

extern "C" int vb_quantize_q8_0(vb_ctx *ctx, const float *x, int64_t K, int64_t M, void *blocks, int rule) {
    VB_REQUIRE(ctx, x && blocks && K > 0 && M >= 0, "vb_quantize_q8_0: bad argument");
    VB_REQUIRE(ctx, rule == VB_QRULE_X86 || rule == VB_QRULE_REF, "vb_quantize_q8_0: unknown rule");
    return launch_quantize_q8_0(ctx, x, K, M, blocks, rule);
}

extern "C" int vb_dequantize_q8_0(vb_ctx *ctx, const void *blocks, int64_t n, float *y) {
    VB_REQUIRE(ctx, blocks && y && n >= 0, "vb_dequantize_q8_0: bad argument");
    return launch_dequantize_q8_0(ctx, blocks, n, y);
}

extern "C" int vb_get_rows(vb_ctx *ctx, vb_weight table, const int32_t *ids, int64_t n, float *y) {
    VB_REQUIRE(ctx, table && ids && y && n >= 0, "vb_get_rows: bad argument");
    return launch_get_rows(ctx, table, ids, n, y);
}

extern "C" int vb_rms_norm(vb_ctx *ctx, const float *x, const float *w, float *y, int64_t n, int64_t rows, float eps,
                           unsigned flags) {
    VB_REQUIRE(ctx, x && y && n > 0 && rows >= 0, "vb_rms_norm: bad argument");
    return launch_rms_norm(ctx, x, w, y, n, rows, eps, flags);
}

extern "C" int vb_bf16_round(vb_ctx *ctx, float *x, int64_t n) {
    VB_REQUIRE(ctx, x && n >= 0, "vb_bf16_round: bad argument");
    return launch_bf16_round(ctx, x, n);
}

extern "C" int vb_residual_add(vb_ctx *ctx, const float *a, const float *b, float scale, float *y, int64_t n,
                               unsigned flags) {
    VB_REQUIRE(ctx, a && b && y && n >= 0, "vb_residual_add: bad argument");
    return launch_residual(ctx, a, b, scale, y, n, flags);
}

extern "C" int vb_swiglu(vb_ctx *ctx, const float *g, const float *u, float *y, int64_t n, unsigned flags) {
    VB_REQUIRE(ctx, g && u && y && n >= 0, "vb_swiglu: bad argument");
    return launch_swiglu(ctx, g, u, y, n, flags);
}

extern "C" int vb_rope_neox(vb_ctx *ctx, float *x, int head_dim, int n_heads, int T, const int32_t *pos, float theta,
                            unsigned flags) {
    VB_REQUIRE(ctx, x && pos && head_dim > 0 && head_dim % 2 == 0 && n_heads > 0 && T >= 0,
               "vb_rope_neox: bad argument");
    // The cos/sin table covers the reference's default max_seq_len (8192).
    const RopeTable *rt = rope_table(ctx, head_dim, theta, head_dim == 128, 8192);
    if (!rt) return VB_ERR_OOM;
    return launch_rope(ctx, x, (int64_t)n_heads * head_dim, head_dim, n_heads, T, pos, rt->d_cs, flags);
}

extern "C" int vb_fsq_quantize(vb_ctx *ctx, float *x, int64_t n, float s) {
    VB_REQUIRE(ctx, x && n >= 0, "vb_fsq_quantize: bad argument");
    return launch_fsq(ctx, x, n, s);
}

extern "C" int vb_attention(vb_ctx *ctx, const float *q, const uint16_t *k, const uint16_t *v, int n_rows, int T,
                            int n_heads, int n_kv_heads, int head_dim, const int32_t *row_start,
                            const int32_t *kv_len, float *out) {
    VB_REQUIRE(ctx, q && k && v && row_start && kv_len && out && n_rows > 0 && T >= 0,
               "vb_attention: bad argument");
    // the grid needs the longest row range; every token range lies in n_rows
    return launch_attention(ctx, q, 0, k, v, n_rows, T, n_heads, n_kv_heads, head_dim, row_start, kv_len, n_rows,
                            out, 0);
}

extern "C" int vb_kv_write(vb_ctx *ctx, const float *k, const float *v, uint16_t *kc, uint16_t *vc, int n_rows, int T,
                           int n_kv_heads, int head_dim, const int32_t *dst_row) {
    VB_REQUIRE(ctx, k && v && kc && vc && dst_row && n_rows > 0 && T >= 0, "vb_kv_write: bad argument");
    return launch_kv_write(ctx, k, v, (int64_t)n_kv_heads * head_dim, kc, vc, n_rows, T, n_kv_heads, head_dim,
                           dst_row);
}
