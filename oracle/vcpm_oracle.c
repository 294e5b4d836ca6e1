/*
 * vcpm_oracle.c -- CPU restatement of VoxCPM-C's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker); see vcpm_oracle.h.
 * Built with -ffp-contract=off so every fp32 expression rounds exactly as
 * written; the CUDA kernels use explicitly rounded intrinsics for the same
 * expressions, which makes the elementwise ops bit-comparable.
 *
 * Reference citations are paths inside the voxcpm-cpp tree.
 */
#include "vcpm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* Accumulator of every dot product (mat-mul blocks, attention scores and
 * value sums).  The default (double) is the most exact restatement; the
 * Makefile also builds liboracle_f32acc.so with VO_ACC=float, which sums in
 * fp32 as ggml-CPU's SIMD lanes do.  Both are the same algorithm up to
 * accumulation order; the distance between their outputs measures how far
 * two legitimate orders drift apart through bf16 casts and Q8_0 activation
 * rounding, and the parity tests calibrate stacked-layer gates with it. */
#ifndef VO_ACC
#define VO_ACC double
#endif

/* ------------------------------------------------------------------------ */
/* scalar conversions                                                        */
/* ------------------------------------------------------------------------ */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* F32 -> BF16, round to nearest even, NaN forced quiet.  This is the
 * conversion behind ggml_cast(F32->BF16) that the reference inserts after
 * every module (src/minicpm4.c:39-42, src/locdit.c:114-121,
 * src/cfm_solver.c:23-25). */
uint16_t vo_fp32_to_bf16(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

float vo_bf16_to_fp32(uint16_t h) { return u2f((uint32_t)h << 16); }

float vo_bf16_round(float x) { return vo_bf16_to_fp32(vo_fp32_to_bf16(x)); }

void vo_bf16_round_array(float *x, int64_t n) {
    for (int64_t i = 0; i < n; i++) x[i] = vo_bf16_round(x[i]);
}

/* IEEE binary16 conversion, round to nearest even (the F16C/_cvtss_sh and
 * numpy float16 rule that ggml uses for Q8_0 scales and F16 operands). */
uint16_t vo_fp32_to_fp16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) {                       /* inf / nan */
        if (a == 0x7f800000u) return sign | 0x7c00u;
        return (uint16_t)(sign | 0x7e00u | ((a >> 13) & 0x3ffu));
    }
    if (a >= 0x477ff000u) return sign | 0x7c00u;  /* >= 65520 rounds to inf */
    if (a < 0x33000000u) return sign;             /* < 2^-25 rounds to zero */
    uint32_t e = a >> 23;
    if (e < 113u) {                               /* half subnormal */
        uint32_t m = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e;                /* 14..24 */
        uint32_t k = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (k & 1u))) k++;
        return (uint16_t)(sign | k);
    }
    uint32_t r = a - (112u << 23);                /* rebias 127 -> 15 */
    uint32_t h = r >> 13;
    uint32_t rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

float vo_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t m = (uint32_t)h & 0x3ffu;
    if (e == 0) {
        if (m == 0) return u2f(sign);
        /* subnormal: m * 2^-24, exact in fp32 */
        float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

static float g_f16_table[65536];
static int g_f16_table_ready = 0;

static void f16_table_init(void) {
    if (g_f16_table_ready) return;
    for (uint32_t i = 0; i < 65536u; i++) g_f16_table[i] = vo_fp16_to_fp32((uint16_t)i);
    g_f16_table_ready = 1;
}

/* ------------------------------------------------------------------------ */
/* Q8_0                                                                      */
/* ------------------------------------------------------------------------ */

typedef struct {
    uint16_t d;
    int8_t qs[VO_QK8_0];
} vo_block_q8_0;

/* Q8_0 quantization of one 32-element block.  Both rules compute the scale
 * d = amax/127 and store it as fp16; they differ in the reciprocal and the
 * tie rule (see vcpm_oracle.h).  The weight rule is what tools/quantize.c:292
 * reaches through ggml_quantize_chunk; the x86 rule is what ggml-CPU applies
 * to the activation rows of every Q8_0 mat-mul (vec_dot_type Q8_0). */
static void quantize_block(const float *x, vo_block_q8_0 *y, int rule) {
    float amax = 0.0f;
    for (int j = 0; j < VO_QK8_0; j++) {
        float a = fabsf(x[j]);
        if (a > amax) amax = a;
    }
    const float d = amax / 127.0f;
    y->d = vo_fp32_to_fp16(d);
    if (rule == VO_QRULE_X86) {
        const float id = (amax != 0.0f) ? 127.0f / amax : 0.0f;
        for (int j = 0; j < VO_QK8_0; j++) {
            float v = rintf(x[j] * id);          /* round half to even */
            y->qs[j] = (int8_t)v;
        }
    } else {
        const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        for (int j = 0; j < VO_QK8_0; j++) {
            float v = roundf(x[j] * id);         /* round half away */
            y->qs[j] = (int8_t)v;
        }
    }
}

void vo_quantize_q8_0(const float *x, void *blocks, int64_t n, int rule) {
    vo_block_q8_0 *y = (vo_block_q8_0 *)blocks;
    for (int64_t b = 0; b < n / VO_QK8_0; b++) quantize_block(x + b * VO_QK8_0, y + b, rule);
}

/* Block dequantization w = qs[j] * fp16->fp32(d), one exact fp32 product
 * (src/model_loader.c:317-331, src/gen_prompt.c:106-125). */
void vo_dequantize_q8_0(const void *blocks, float *y, int64_t n) {
    const vo_block_q8_0 *x = (const vo_block_q8_0 *)blocks;
    for (int64_t b = 0; b < n / VO_QK8_0; b++) {
        const float d = vo_fp16_to_fp32(x[b].d);
        for (int j = 0; j < VO_QK8_0; j++) y[b * VO_QK8_0 + j] = (float)x[b].qs[j] * d;
    }
}

/* Embedding lookup of gen_forward_text (src/gen_prompt.c:67-131): out row
 * i = table row ids[i] as F32, an id outside [0, n_rows) reading row 0.
 * Q8_0 values are qs * fp16->fp32(d) (:106-125), F16 the exact widening
 * (:88-95), F32 a copy (:96-103).  Returns -1 for an unknown type. */
int vo_get_rows(int type, const void *table, int64_t K, int64_t n_rows, const int32_t *ids, int64_t n,
                float *out) {
    const size_t rb = vo_row_bytes(type, K);
    if (rb == 0) return -1;
    for (int64_t i = 0; i < n; i++) {
        int64_t id = ids[i];
        if (id < 0 || id >= n_rows) id = 0;
        const uint8_t *row = (const uint8_t *)table + (size_t)id * rb;
        float *y = out + i * K;
        if (type == VO_TYPE_Q8_0) {
            vo_dequantize_q8_0(row, y, K);
        } else if (type == VO_TYPE_F16) {
            const uint16_t *h = (const uint16_t *)row;
            for (int64_t k = 0; k < K; k++) y[k] = vo_fp16_to_fp32(h[k]);
        } else {
            memcpy(y, row, (size_t)K * 4u);
        }
    }
    return 0;
}

size_t vo_row_bytes(int type, int64_t K) {
    switch (type) {
    case VO_TYPE_F32: return (size_t)K * 4u;
    case VO_TYPE_F16: return (size_t)K * 2u;
    case VO_TYPE_Q8_0: return (size_t)(K / VO_QK8_0) * VO_Q8_0_BYTES;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* mat-mul: ggml_mul_mat(W[K,N], x[K,M]) -> y[N,M]                           */
/* ------------------------------------------------------------------------ */

/* Q8_0 x Q8_0 block dot: per block the exact int32 sum of 32 products,
 * scaled by the fp32 product of the two fp16 scales; blocks accumulate in
 * double (ggml accumulates in fp32 lanes; the difference is accumulation
 * order only). */
static float dot_q8_0(const vo_block_q8_0 *w, const vo_block_q8_0 *x, int64_t nb) {
    VO_ACC acc = 0.0;
    for (int64_t b = 0; b < nb; b++) {
        int32_t s = 0;
        for (int j = 0; j < VO_QK8_0; j++) s += (int32_t)w[b].qs[j] * (int32_t)x[b].qs[j];
        const float d = g_f16_table[w[b].d] * g_f16_table[x[b].d];
        acc += (double)((float)s * d);
    }
    return (float)acc;
}

static float dot_f16(const uint16_t *w, const uint16_t *x, int64_t K) {
    VO_ACC acc = 0.0;
    for (int64_t k = 0; k < K; k++) acc += (double)(g_f16_table[w[k]] * g_f16_table[x[k]]);
    return (float)acc;
}

static float dot_f32(const float *w, const float *x, int64_t K) {
    VO_ACC acc = 0.0;
    for (int64_t k = 0; k < K; k++) acc += (double)(w[k] * x[k]);
    return (float)acc;
}

int vo_matmul(int wtype, const void *W, int64_t K, int64_t N, const float *x,
              int64_t M, float *y, int qrule, int nthreads) {
    if (!W || !x || !y || K <= 0 || N <= 0 || M < 0) return -1;
    if (M == 0) return 0;
    f16_table_init();
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
    (void)nthreads;
#endif
    if (wtype == VO_TYPE_Q8_0) {
        if (K % VO_QK8_0) return -1;
        const int64_t nb = K / VO_QK8_0;
        vo_block_q8_0 *xq = (vo_block_q8_0 *)malloc((size_t)(M * nb) * sizeof(vo_block_q8_0));
        if (!xq) return -1;
        for (int64_t m = 0; m < M; m++) vo_quantize_q8_0(x + m * K, xq + m * nb, K, qrule);
        const vo_block_q8_0 *wb = (const vo_block_q8_0 *)W;
#ifdef _OPENMP
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
        for (int64_t n = 0; n < N; n++)
            for (int64_t m = 0; m < M; m++) y[m * N + n] = dot_q8_0(wb + n * nb, xq + m * nb, nb);
        free(xq);
    } else if (wtype == VO_TYPE_F16) {
        uint16_t *xh = (uint16_t *)malloc((size_t)(M * K) * 2u);
        if (!xh) return -1;
        for (int64_t i = 0; i < M * K; i++) xh[i] = vo_fp32_to_fp16(x[i]);
        const uint16_t *wh = (const uint16_t *)W;
#ifdef _OPENMP
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
        for (int64_t n = 0; n < N; n++)
            for (int64_t m = 0; m < M; m++) y[m * N + n] = dot_f16(wh + n * K, xh + m * K, K);
        free(xh);
    } else if (wtype == VO_TYPE_F32) {
        const float *wf = (const float *)W;
#ifdef _OPENMP
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
        for (int64_t n = 0; n < N; n++)
            for (int64_t m = 0; m < M; m++) y[m * N + n] = dot_f32(wf + n * K, x + m * K, K);
    } else {
        return -1;
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* elementwise ops                                                           */
/* ------------------------------------------------------------------------ */

/* ggml_rms_norm: fp32 squares summed in double, mean narrowed to fp32,
 * scale = 1/sqrtf(mean+eps), y = x*scale. */
void vo_rms_norm(const float *x, float *y, int64_t n, int64_t rows, float eps) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * n;
        float *yr = y + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; i++) sum += (double)(xr[i] * xr[i]);
        const float mean = (float)(sum / (double)n);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < n; i++) yr[i] = xr[i] * scale;
    }
}

/* vcpm_rms_norm (src/minicpm4.c:132-152): bf16(bf16(rms_norm(x)) * w). */
void vo_rms_norm_bf16(const float *x, const float *w, float *y, int64_t n,
                      int64_t rows, float eps) {
    vo_rms_norm(x, y, n, rows, eps);
    for (int64_t r = 0; r < rows; r++)
        for (int64_t i = 0; i < n; i++)
            y[r * n + i] = vo_bf16_round(vo_bf16_round(y[r * n + i]) * w[i]);
}

float vo_silu(float x) { return x / (1.0f + expf(-x)); }

/* vcpm_fsq_quantize (src/fsq.c:16-29): tanh -> *s -> round -> *(1/s). */
void vo_fsq_quantize(float *x, int64_t n, float quant_scale) {
    if (quant_scale <= 0.0f) return;
    const float inv = 1.0f / quant_scale;
    for (int64_t i = 0; i < n; i++) x[i] = roundf(tanhf(x[i]) * quant_scale) * inv;
}

/* VoxCPM2 LongRoPE short factors: model configuration data (one divisor per
 * rotary pair), applied when head_dim == 128 (src/minicpm4.c:49-66,183-188). */
static const float k_longrope_short[64] = {
    0.9977997200f, 1.0146582960f, 1.0349680405f, 1.0594292461f,
    1.0888815017f, 1.1243301355f, 1.1669771036f, 1.2182568067f,
    1.2798772354f, 1.3538666752f, 1.4426259040f, 1.5489853360f,
    1.6762658237f, 1.8283407612f, 2.0096956086f, 2.2254789275f,
    2.4815363797f, 2.7844159346f, 3.1413289096f, 3.5600478448f,
    4.0487193801f, 4.6155695421f, 5.2684819497f, 6.0144385919f,
    6.8588300492f, 7.8046682500f, 8.8517684937f, 9.9960050583f,
    11.2287664413f, 12.5367574692f, 13.9022579193f, 15.3038854599f,
    16.7178382874f, 18.1194648743f, 19.4849643707f, 20.7929573059f,
    22.0257186890f, 23.1699542999f, 24.2170543671f, 25.1628932953f,
    26.0072841644f, 26.7532405853f, 27.4061527252f, 27.9730033875f,
    28.4616756439f, 28.8803939819f, 29.2373065948f, 29.5401859283f,
    29.7962436676f, 30.0120277405f, 30.1933822632f, 30.3454570770f,
    30.4727382660f, 30.5790977478f, 30.6678562164f, 30.7418460846f,
    30.8034667969f, 30.8547458649f, 30.8973922729f, 30.9328403473f,
    30.9622936249f, 30.9867553711f, 31.0070648193f, 31.0239238739f,
};

const float *vo_longrope_short_factors(void) { return k_longrope_short; }

/* cos/sin of the NEOX rotary angles for one position, as ggml_rope_ext
 * builds them with freq_scale=1, ext_factor=0, attn_factor=1: the angle of
 * pair i is theta_i/ff_i where theta_0 = pos and theta_{i+1} =
 * theta_i * base^(-2/head_dim) in fp32 (src/minicpm4.c:205-213).
 * cs[2i] = cos, cs[2i+1] = sin. */
void vo_rope_cache(float *cs, int32_t pos, int head_dim, float theta_base,
                   const float *freq_factors) {
    const float theta_scale = powf(theta_base, -2.0f / (float)head_dim);
    float theta = (float)pos;
    for (int i0 = 0; i0 < head_dim; i0 += 2) {
        const float ff = freq_factors ? freq_factors[i0 / 2] : 1.0f;
        const float a = theta / ff;
        cs[i0] = cosf(a);
        cs[i0 + 1] = sinf(a);
        theta *= theta_scale;
    }
}

/* NEOX rotation of x[T][n_heads][head_dim] in place: pair i couples
 * element i with element i + head_dim/2. */
void vo_rope_neox(float *x, int head_dim, int n_heads, int n_tokens,
                  int32_t pos0, float theta, const float *freq_factors) {
    float *cs = (float *)malloc((size_t)head_dim * sizeof(float));
    const int half = head_dim / 2;
    for (int t = 0; t < n_tokens; t++) {
        vo_rope_cache(cs, pos0 + t, head_dim, theta, freq_factors);
        for (int h = 0; h < n_heads; h++) {
            float *v = x + ((size_t)t * n_heads + h) * head_dim;
            for (int i = 0; i < half; i++) {
                const float c = cs[2 * i], s = cs[2 * i + 1];
                const float x0 = v[i], x1 = v[i + half];
                v[i] = x0 * c - x1 * s;
                v[i + half] = x0 * s + x1 * c;
            }
        }
    }
    free(cs);
}

/* ------------------------------------------------------------------------ */
/* transformer                                                               */
/* ------------------------------------------------------------------------ */

static void maybe_bf16(float *x, int64_t n, const vo_opts *o) {
    if (o->bf16) vo_bf16_round_array(x, n);
}

/* ggml_soft_max_ext(scale=1, no mask) over n scores: max-subtracted expf,
 * sum in double, then multiply by (float)(1/sum). */
static void softmax_inplace(float *s, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) if (s[i] > mx) mx = s[i];
    double sum = 0.0;
    for (int i = 0; i < n; i++) { s[i] = expf(s[i] - mx); sum += (double)s[i]; }
    const float inv = (float)(1.0 / sum);
    for (int i = 0; i < n; i++) s[i] *= inv;
}

/* vcpm_attention (src/minicpm4.c:250-428) with gqa_group_attn (:232-248). */
int vo_attention(const vo_lm_config *cfg, const vo_layer_weights *w,
                 vo_kv_layer *cache, const float *x, int T, int pos,
                 int no_causal, float *out, const vo_opts *o) {
    const int H = cfg->hidden, NH = cfg->n_heads, NKV = cfg->n_kv_heads, HD = cfg->head_dim;
    const int QD = NH * HD, KD = NKV * HD, QPK = NH / NKV;
    if (!no_causal && !cache) return -1;
    float *q = (float *)malloc((size_t)T * QD * 4);
    float *k = (float *)malloc((size_t)T * KD * 4);
    float *v = (float *)malloc((size_t)T * KD * 4);
    float *att = (float *)malloc((size_t)T * QD * 4);
    int kvmax = no_causal ? T : cache->n_used + T;
    float *sc = (float *)malloc((size_t)(kvmax > 0 ? kvmax : 1) * 4);
    if (!q || !k || !v || !att || !sc) return -1;

    vo_matmul(w->wtype, w->q, H, QD, x, T, q, o->qrule, o->nthreads);
    maybe_bf16(q, (int64_t)T * QD, o);
    vo_matmul(w->wtype, w->k, H, KD, x, T, k, o->qrule, o->nthreads);
    maybe_bf16(k, (int64_t)T * KD, o);
    vo_matmul(w->wtype, w->v, H, KD, x, T, v, o->qrule, o->nthreads);
    maybe_bf16(v, (int64_t)T * KD, o);

    if (!cfg->no_rope) {
        const float *ff = (HD == 128) ? k_longrope_short : NULL;
        vo_rope_neox(q, HD, NH, T, pos, cfg->rope_theta, ff);
        vo_rope_neox(k, HD, NKV, T, pos, cfg->rope_theta, ff);
        maybe_bf16(q, (int64_t)T * QD, o);
        maybe_bf16(k, (int64_t)T * KD, o);
    }

    int write_pos = 0;
    if (cache) {
        write_pos = cache->n_used;
        if (write_pos + T > cache->capacity) return -1;
        memcpy(cache->k + (size_t)write_pos * KD, k, (size_t)T * KD * 4);
        memcpy(cache->v + (size_t)write_pos * KD, v, (size_t)T * KD * 4);
        cache->n_used = write_pos + T;
    }

    const float kq_scale = 1.0f / sqrtf((float)HD);
    for (int ti = 0; ti < T; ti++) {
        const float *ks, *vs;
        int L;
        if (no_causal) { ks = k; vs = v; L = T; }
        else { ks = cache->k; vs = cache->v; L = write_pos + ti + 1; }
        for (int g = 0; g < NKV; g++) {
            for (int j = 0; j < QPK; j++) {
                const int h = g * QPK + j;
                const float *qv = q + (size_t)ti * QD + (size_t)h * HD;
                for (int l = 0; l < L; l++) {
                    const float *kv = ks + (size_t)l * KD + (size_t)g * HD;
                    VO_ACC acc = 0.0;
                    for (int d = 0; d < HD; d++) acc += (double)(kv[d] * qv[d]);
                    sc[l] = (float)acc * kq_scale;
                }
                softmax_inplace(sc, L);
                float *ov = att + (size_t)ti * QD + (size_t)h * HD;
                for (int d = 0; d < HD; d++) {
                    VO_ACC acc = 0.0;
                    for (int l = 0; l < L; l++) acc += (double)(vs[(size_t)l * KD + (size_t)g * HD + d] * sc[l]);
                    ov[d] = (float)acc;
                }
            }
        }
    }
    /* o_proj per token (src/minicpm4.c:415); column-independent, so one
     * batched mat-mul gives the same values. */
    vo_matmul(w->wtype, w->o, QD, H, att, T, out, o->qrule, o->nthreads);
    maybe_bf16(out, (int64_t)T * H, o);
    free(q); free(k); free(v); free(att); free(sc);
    return 0;
}

/* vcpm_mlp (src/minicpm4.c:432-463). With o->bf16 == 0 it is the raw
 * silu(gate x) * (up x) -> down graph of tests/test_fixture_parity.c. */
int vo_mlp(int wtype, const void *gate, const void *up, const void *down,
           int hidden, int ffn, const float *x, int T, float *out,
           const vo_opts *o) {
    float *g = (float *)malloc((size_t)T * ffn * 4);
    float *u = (float *)malloc((size_t)T * ffn * 4);
    if (!g || !u) return -1;
    vo_matmul(wtype, gate, hidden, ffn, x, T, g, o->qrule, o->nthreads);
    maybe_bf16(g, (int64_t)T * ffn, o);
    for (int64_t i = 0; i < (int64_t)T * ffn; i++) g[i] = vo_silu(g[i]);
    maybe_bf16(g, (int64_t)T * ffn, o);
    vo_matmul(wtype, up, hidden, ffn, x, T, u, o->qrule, o->nthreads);
    maybe_bf16(u, (int64_t)T * ffn, o);
    for (int64_t i = 0; i < (int64_t)T * ffn; i++) g[i] = g[i] * u[i];
    maybe_bf16(g, (int64_t)T * ffn, o);
    vo_matmul(wtype, down, ffn, hidden, g, T, out, o->qrule, o->nthreads);
    maybe_bf16(out, (int64_t)T * hidden, o);
    free(g); free(u);
    return 0;
}

/* vcpm_minicpm4_block (src/minicpm4.c:467-532), h[T][hidden] in place. */
int vo_block(const vo_lm_config *cfg, const vo_layer_weights *w,
             vo_kv_layer *cache, float *h, int T, int pos, int no_causal,
             float scale, const vo_opts *o) {
    const int H = cfg->hidden;
    const int64_t n = (int64_t)T * H;
    float *xn = (float *)malloc((size_t)n * 4);
    float *a = (float *)malloc((size_t)n * 4);
    if (!xn || !a) return -1;
    vo_rms_norm_bf16(h, w->attn_norm, xn, H, T, cfg->eps);
    if (vo_attention(cfg, w, cache, xn, T, pos, no_causal, a, o)) return -1;
    for (int64_t i = 0; i < n; i++) {
        const float s = (scale != 1.0f) ? a[i] * scale : a[i];
        h[i] = vo_bf16_round(h[i] + s);
    }
    vo_rms_norm_bf16(h, w->ffn_norm, xn, H, T, cfg->eps);
    if (vo_mlp(w->wtype, w->gate, w->up, w->down, H, cfg->ffn, xn, T, a, o)) return -1;
    for (int64_t i = 0; i < n; i++) {
        const float s = (scale != 1.0f) ? a[i] * scale : a[i];
        h[i] = vo_bf16_round(h[i] + s);
    }
    free(xn); free(a);
    return 0;
}

/* vcpm_minicpm4_forward (src/minicpm4.c:536-572). */
int vo_lm_forward(const vo_lm_config *cfg, const vo_layer_weights *layers,
                  const float *final_norm, vo_kv_layer *caches,
                  const float *x, int T, int pos, float *out,
                  const vo_opts *o) {
    const int64_t n = (int64_t)T * cfg->hidden;
    float *h = (float *)malloc((size_t)n * 4);
    if (!h) return -1;
    memcpy(h, x, (size_t)n * 4);
    float scale = 1.0f;
    if (cfg->scale_depth > 0.0f && cfg->n_layers > 0)
        scale = cfg->scale_depth / sqrtf((float)cfg->n_layers);
    for (int l = 0; l < cfg->n_layers; l++)
        if (vo_block(cfg, &layers[l], &caches[l], h, T, pos, 0, scale, o)) { free(h); return -1; }
    vo_rms_norm_bf16(h, final_norm, out, cfg->hidden, T, cfg->eps);
    free(h);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* LocDiT (src/locdit.c)                                                     */
/* ------------------------------------------------------------------------ */

/* dit_sinusoidal_t_embed (src/locdit.c:163-188): [sin(half) | cos(half)]. */
void vo_dit_time_sin(float t, int dim, float *out) {
    const int half = dim / 2;
    const float log_max_period = logf(10000.0f);
    const float denom = (half > 1) ? (float)(half - 1) : 1.0f;
    const float scaled_t = vo_bf16_round(t * 1000.0f);
    for (int i = 0; i < half; i++) {
        const float exponent = vo_bf16_round(vo_bf16_round((float)i) * (-log_max_period / denom));
        const float freq = vo_bf16_round(expf(exponent));
        const float angle = vo_bf16_round(freq * scaled_t);
        out[i] = vo_bf16_round(sinf(angle));
        out[half + i] = vo_bf16_round(cosf(angle));
    }
}

static void linear_bias(int wtype, const void *W, const float *b, int K, int N,
                        const float *x, int T, float *y, const vo_opts *o) {
    vo_matmul(wtype, W, K, N, x, T, y, o->qrule, o->nthreads);
    if (b)
        for (int t = 0; t < T; t++)
            for (int n = 0; n < N; n++) y[(size_t)t * N + n] = y[(size_t)t * N + n] + b[n];
}

/* vcpm_time_mlp_forward (src/locdit.c:140-159). */
static void time_mlp(int wtype, const void *w1, const float *b1, const void *w2,
                     const float *b2, int H, const float *tsin, float *out,
                     const vo_opts *o) {
    float *h = (float *)malloc((size_t)H * 4);
    linear_bias(wtype, w1, b1, H, H, tsin, 1, h, o);
    for (int i = 0; i < H; i++) h[i] = vo_bf16_round(vo_silu(vo_bf16_round(h[i])));
    linear_bias(wtype, w2, b2, H, H, h, 1, out, o);
    vo_bf16_round_array(out, H);
    free(h);
}

/* vcpm_locdit_forward (src/locdit.c:216-400).  x, cond: [P][feat]; mu:
 * [2*hidden] or NULL (unconditional branch, zero tokens); out: [P][feat]. */
int vo_dit_forward(const vo_dit_config *cfg, const vo_dit_weights *w,
                   const float *x, const float *cond, float t, float dt,
                   const float *mu, float *out, const vo_opts *o) {
    const int H = cfg->hidden, P = cfg->patch, F = cfg->feat_dim;
    const int T = 3 + 2 * P;
    float *seq = (float *)calloc((size_t)T * H, 4);
    float *tsin = (float *)malloc((size_t)H * 4);
    float *tf = (float *)malloc((size_t)H * 4);
    float *dtf = (float *)malloc((size_t)H * 4);
    if (!seq || !tsin || !tf || !dtf) return -1;

    /* tokens 3+P .. 3+2P-1: bf16(in_proj(x) + b) */
    linear_bias(w->wtype, w->in_proj, w->in_bias, F, H, x, P, seq + (size_t)(3 + P) * H, o);
    vo_bf16_round_array(seq + (size_t)(3 + P) * H, (int64_t)P * H);
    /* tokens 3 .. 3+P-1: bf16(cond_proj(cond) + b) */
    linear_bias(w->wtype, w->cond_proj, w->cond_bias, F, H, cond, P, seq + (size_t)3 * H, o);
    vo_bf16_round_array(seq + (size_t)3 * H, (int64_t)P * H);
    /* token 2: bf16(time_mlp(t) + delta_time_mlp(dt)) */
    vo_dit_time_sin(t, H, tsin);
    time_mlp(w->wtype, w->t_w1, w->t_b1, w->t_w2, w->t_b2, H, tsin, tf, o);
    vo_dit_time_sin(dt, H, tsin);
    time_mlp(w->wtype, w->dt_w1, w->dt_b1, w->dt_w2, w->dt_b2, H, tsin, dtf, o);
    for (int i = 0; i < H; i++) seq[(size_t)2 * H + i] = vo_bf16_round(tf[i] + dtf[i]);
    /* tokens 0, 1: mu halves (raw fp32), or zeros */
    if (mu) memcpy(seq, mu, (size_t)2 * H * 4);

    vo_lm_config lc;
    lc.hidden = H; lc.n_heads = cfg->n_heads; lc.n_kv_heads = cfg->n_kv_heads;
    lc.head_dim = cfg->head_dim; lc.ffn = cfg->ffn; lc.n_layers = cfg->n_layers;
    lc.eps = cfg->eps; lc.rope_theta = 10000.0f; lc.no_rope = 0; lc.scale_depth = 0.0f;
    for (int l = 0; l < cfg->n_layers; l++)
        if (vo_block(&lc, &w->layers[l], NULL, seq, T, 0, 1, 1.0f, o)) return -1;

    float *hn = (float *)malloc((size_t)P * H * 4);
    vo_rms_norm_bf16(seq + (size_t)(3 + P) * H, w->norm, hn, H, P, cfg->eps);
    linear_bias(w->wtype, w->out_proj, w->out_bias, H, F, hn, P, out, o);
    vo_bf16_round_array(out, (int64_t)P * F);
    free(seq); free(tsin); free(tf); free(dtf); free(hn);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* LocEnc (src/locenc.c:44-131)                                              */
/* ------------------------------------------------------------------------ */

int vo_enc_forward(const vo_enc_config *cfg, const vo_enc_weights *w,
                   const float *patch, int P, float *cls_out,
                   const vo_opts *o) {
    const int H = cfg->hidden, T = P + 1;
    float *seq = (float *)malloc((size_t)T * H * 4);
    if (!seq) return -1;
    memcpy(seq, w->special, (size_t)H * 4);
    linear_bias(w->wtype, w->in_proj, w->in_bias, cfg->feat_dim, H, patch, P, seq + H, o);
    vo_lm_config lc;
    lc.hidden = H; lc.n_heads = cfg->n_heads; lc.n_kv_heads = cfg->n_kv_heads;
    lc.head_dim = cfg->head_dim; lc.ffn = cfg->ffn; lc.n_layers = cfg->n_layers;
    lc.eps = cfg->eps; lc.rope_theta = 10000.0f; lc.no_rope = 0; lc.scale_depth = 0.0f;
    for (int l = 0; l < cfg->n_layers; l++)
        if (vo_block(&lc, &w->layers[l], NULL, seq, T, 0, 1, 1.0f, o)) { free(seq); return -1; }
    vo_rms_norm_bf16(seq, w->norm, cls_out, H, 1, cfg->eps);
    free(seq);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* CFM                                                                       */
/* ------------------------------------------------------------------------ */

/* vcpm_cfm_sway_t_bf16 (src/cfm_solver.c:27-37). */
float vo_cfm_sway_t_bf16(int step, int n_steps) {
    if (n_steps <= 0 || step < 0 || step > n_steps) return 0.0f;
    const float base = vo_bf16_round(1.0f - (float)step / (float)n_steps);
    const float half_pi = vo_bf16_round(1.57079632679489661923f);
    const float angle = vo_bf16_round(half_pi * base);
    const float cosine = vo_bf16_round(cosf(angle));
    const float inner = vo_bf16_round(vo_bf16_round(cosine - 1.0f) + base);
    return vo_bf16_round(base + inner);
}

/* vcpm_cfm_cfg_zero_star (src/cfm_solver.c:65-93): writes the guided
 * velocity into `negative` and returns st*. */
float vo_cfg_zero_star(float *negative, const float *positive, int n, float cfg_value) {
    if (!negative || !positive || n <= 0) return 1.0f;
    double dot = 0.0, sq = 0.0;
    for (int i = 0; i < n; i++) {
        const float p = vo_bf16_round(positive[i]);
        const float q = vo_bf16_round(negative[i]);
        dot += vo_bf16_round(p * q);
        sq += vo_bf16_round(q * q);
    }
    const float dot_b = vo_bf16_round((float)dot);
    const float norm_b = vo_bf16_round((float)sq + 1.0e-8f);
    const float st = vo_bf16_round(dot_b / norm_b);
    const float cfg_b = vo_bf16_round(cfg_value);
    for (int i = 0; i < n; i++) {
        const float p = vo_bf16_round(positive[i]);
        const float q = vo_bf16_round(negative[i]);
        const float qs = vo_bf16_round(q * st);
        const float delta = vo_bf16_round(p - qs);
        const float guide = vo_bf16_round(cfg_b * delta);
        negative[i] = vo_bf16_round(qs + guide);
    }
    return st;
}

/* vcpm_cfm_zero_star_steps (src/gen_step.c:50-54). */
int vo_cfm_zero_star_steps(int n_steps) {
    if (n_steps <= 1) return 0;
    int z = (int)(((float)n_steps + 1.0f) * 0.04f);
    return z > 1 ? z : 1;
}

/* SplitMix64 + Box-Muller draw used for CFM noise (src/gen_step.c:409-431). */
static uint64_t splitmix_next(uint64_t *s) {
    *s += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static float box_muller(uint64_t *s) {
    float u1 = (float)(splitmix_next(s) >> 11) * (1.0f / 9007199254740992.0f);
    u1 = fmaxf(1e-6f, fminf(u1, 1.0f - 1e-6f));
    float u2 = (float)(splitmix_next(s) >> 11) * (1.0f / 9007199254740992.0f);
    u2 = fmaxf(1e-6f, fminf(u2, 1.0f - 1e-6f));
    return sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265358979323846f * u2);
}

void vo_cfm_noise(uint64_t seed, int ar_step, float *x, int n) {
    uint64_t s = seed ^ ((uint64_t)(ar_step + 1) * 0xD2B74407B1CE6E93ULL);
    for (int j = 0; j < n; j++) x[j] = vo_bf16_round(box_muller(&s));
}

void vo_fill_normal(uint64_t seed, float mean, float stddev, float *x, int64_t n) {
    uint64_t s = seed * 0x9E3779B97F4A7C15ULL + 0x632BE59BD9B4E019ULL;
    for (int64_t i = 0; i < n; i++) x[i] = mean + stddev * box_muller(&s);
}

/* The Euler CFM loop of vcpm_gen_step (src/gen_step.c:472-652). */
int vo_cfm_solve(const vo_dit_config *cfg, const vo_dit_weights *w,
                 const float *mu, const float *cond, float *x, int n_steps,
                 float cfg_value, const vo_opts *o) {
    const int n = cfg->patch * cfg->feat_dim;
    const int zero_star = vo_cfm_zero_star_steps(n_steps);
    const int use_cfg = (cfg_value != 1.0f && mu != NULL);
    float *vc = (float *)malloc((size_t)n * 4);
    float *vu = (float *)malloc((size_t)n * 4);
    if (!vc || !vu) return -1;
    for (int step = 0; step < n_steps; step++) {
        if (step < zero_star) continue;
        const float t = vo_cfm_sway_t_bf16(step, n_steps);
        const float nt = vo_cfm_sway_t_bf16(step + 1, n_steps);
        const float step_size = vo_bf16_round(-(t - nt));
        if (vo_dit_forward(cfg, w, x, cond, t, 0.0f, mu, vc, o)) return -1;
        const float *vel = vc;
        if (use_cfg) {
            if (vo_dit_forward(cfg, w, x, cond, t, 0.0f, NULL, vu, o)) return -1;
            vo_cfg_zero_star(vu, vc, n, cfg_value);
            vel = vu;
        }
        for (int j = 0; j < n; j++) {
            const float delta = vo_bf16_round(step_size * vel[j]);
            x[j] = vo_bf16_round(x[j] + delta);
        }
    }
    free(vc); free(vu);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Stop predictor (src/gen_stop.c:28-230)                                    */
/* ------------------------------------------------------------------------ */

/* read_tensor_f32 (src/gen_stop.c:28-74): the flat tensor as F32 -- F16 the
 * exact widening, Q8_0 (float)qs * fp16->fp32(d) per 34-byte block, F32 a
 * copy.  Returns 0, or -1 for another type. */
static int stop_read_f32(int type, const void *t, float *dst, size_t n) {
    if (type == VO_TYPE_F32) {
        memcpy(dst, t, n * 4u);
        return 0;
    }
    if (type == VO_TYPE_F16) {
        const uint16_t *h = (const uint16_t *)t;
        for (size_t i = 0; i < n; i++) dst[i] = vo_fp16_to_fp32(h[i]);
        return 0;
    }
    if (type == VO_TYPE_Q8_0) {
        if (n % VO_QK8_0) return -1;
        vo_dequantize_q8_0(t, dst, (int64_t)n);
        return 0;
    }
    return -1;
}

/* gen_predict_stop (src/gen_stop.c:85-230) on one hidden row of hs values:
 *   proj[i]  = bias[i] + sum_j W[j*hs + i] * hidden[j]   (stop_proj read in
 *              its [in][out] storage order, :126-137, bias first)
 *   proj[i]  = proj[i] / (1 + expf(-proj[i]))             (fp32 SiLU, :174-178)
 *   logit[o] = sum_j H[2*j + o] * proj[j]                 (stop_head, no bias,
 *              stride 2, :180-200)
 * and the class with torch.argmax's tie rule (class 0 wins ties,
 * gen_stop_class_from_logits :76-81).  The reference accumulates in fp32
 * sequentially; VO_ACC is that order's accumulator (float in the
 * fp32-accumulation build, which is then the reference's exact op order).
 * Returns the class, or -1 on a bad argument. */
int vo_stop_predict(int proj_type, const void *proj_w, const float *proj_bias, int head_type, const void *head_w,
                    const float *hidden, int hs, float *logits) {
    if (!proj_w || !head_w || !hidden || !logits || hs <= 0) return -1;
    float *W = (float *)malloc((size_t)hs * hs * 4u);
    float *Hh = (float *)malloc((size_t)hs * 2u * 4u);
    float *proj = (float *)malloc((size_t)hs * 4u);
    int rc = (W && Hh && proj) ? 0 : -1;
    if (!rc) rc = stop_read_f32(proj_type, proj_w, W, (size_t)hs * hs);
    if (!rc) rc = stop_read_f32(head_type, head_w, Hh, (size_t)hs * 2u);
    if (!rc) {
        for (int i = 0; i < hs; i++) {
            VO_ACC sum = proj_bias ? proj_bias[i] : 0.0f;
            for (int j = 0; j < hs; j++) sum += W[(size_t)j * hs + i] * hidden[j];
            proj[i] = (float)sum;
        }
        for (int i = 0; i < hs; i++) {
            const float x = proj[i];
            proj[i] = x / (1.0f + expf(-x));
        }
        VO_ACC s0 = 0.0f, s1 = 0.0f;
        for (int j = 0; j < hs; j++) {
            s0 += Hh[2 * j + 0] * proj[j];
            s1 += Hh[2 * j + 1] * proj[j];
        }
        logits[0] = (float)s0;
        logits[1] = (float)s1;
        rc = logits[1] > logits[0] ? 1 : 0;
    }
    free(W);
    free(Hh);
    free(proj);
    return rc;
}

/* vcpm_gen_round_cache_capacity (src/gen_init.c:115-127). */
int vo_round_cache_capacity(int required, int model_max) {
    if (required <= 0 || model_max <= 0 || required > model_max) return 0;
    int capacity = 128;
    while (capacity < required) {
        if (capacity > model_max / 2) { capacity = model_max; break; }
        capacity *= 2;
    }
    return capacity <= model_max ? capacity : model_max;
}
