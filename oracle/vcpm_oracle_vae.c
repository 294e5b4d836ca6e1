/*
 * vcpm_oracle_vae.c -- CPU restatement of the AudioVAE V2 decoder, batch and
 * streaming.  TEST INFRASTRUCTURE ONLY (see vcpm_oracle.h).
 *
 * Follows the graph the reference builds in src/audio_vae_stream.c:184-619
 * (streaming, per-layer history caches) and src/audio_vae_v2_decoder.c:149-282
 * (whole-utterance decode with causal zero padding), with the layer helpers
 * of src/audio_vae_v2.c:
 *   conv1d_layer / depthwise_conv1d   :214-407   causal conv, bias added after
 *   upconv_transpose1d                :409-441   transposed conv, causal trim
 *   snake_activation                  :483-503   x + sin(a*x)^2 / a, one op at a time
 *   residual_unit                     :567-636   snake, depthwise k7, snake, pointwise, skip
 *   decoder block table               :40-43     channels D>>b -> D>>(b+1), kernel 2*stride
 * Tensors are kept time-major here ([time][channels]); ggml stores them
 * channel-major, which changes no value.  Every elementwise op is one fp32
 * operation (compiled with -ffp-contract=off), as ggml's separate graph
 * nodes are; dot products accumulate in VO_ACC and are rounded to fp32 once.
 *
 * A whole-utterance decode equals a streaming decode from zeroed caches: the
 * reference pads every causal conv with zeros on the left and the streaming
 * caches start zeroed (src/audio_vae_stream.c:37-49).
 */
#include "vcpm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#ifndef VO_ACC
#define VO_ACC double
#endif

static const int vo_vae_dil[3] = {1, 3, 9};

struct vo_vae_stream {
    vo_vae_config cfg;
    const float *const *w;      /* VO_VAE_* slots */
    float *cache_in;            /* [6][latent]  model.0 history */
    float *cache_up[6];         /* [1][Ci]      upconv history */
    float *cache_res[6][3];     /* [6*d][Co]    depthwise history */
    float *cache_out;           /* [6][C_last]  model.9 history */
};

static int vo_vae_channels(const vo_vae_config *c, int level) { return c->decoder_dim >> level; }

int vo_vae_check_config(const vo_vae_config *c) {
    if (!c || c->latent_dim <= 0 || c->decoder_dim <= 0 || (c->decoder_dim % 64) != 0) return -1;
    for (int i = 0; i < 6; i++)
        if (c->rates[i] <= 0) return -1;
    return 0;
}

int vo_vae_upsample(const vo_vae_config *c) {
    int f = 1;
    for (int i = 0; i < 6; i++) f *= c->rates[i];
    return f;
}

vo_vae_stream *vo_vae_stream_create(const vo_vae_config *cfg, const float *const *w) {
    if (vo_vae_check_config(cfg) || !w) return NULL;
    vo_vae_stream *s = (vo_vae_stream *)calloc(1, sizeof(*s));
    if (!s) return NULL;
    s->cfg = *cfg;
    s->w = w;
    int ok = 1;
    s->cache_in = (float *)calloc((size_t)6 * cfg->latent_dim, sizeof(float));
    ok &= s->cache_in != NULL;
    for (int b = 0; b < 6; b++) {
        const int ci = vo_vae_channels(cfg, b), co = vo_vae_channels(cfg, b + 1);
        s->cache_up[b] = (float *)calloc((size_t)ci, sizeof(float));
        ok &= s->cache_up[b] != NULL;
        for (int r = 0; r < 3; r++) {
            s->cache_res[b][r] = (float *)calloc((size_t)6 * vo_vae_dil[r] * co, sizeof(float));
            ok &= s->cache_res[b][r] != NULL;
        }
    }
    s->cache_out = (float *)calloc((size_t)6 * vo_vae_channels(cfg, 6), sizeof(float));
    ok &= s->cache_out != NULL;
    if (!ok) {
        vo_vae_stream_free(s);
        return NULL;
    }
    return s;
}

void vo_vae_stream_free(vo_vae_stream *s) {
    if (!s) return;
    free(s->cache_in);
    for (int b = 0; b < 6; b++) {
        free(s->cache_up[b]);
        for (int r = 0; r < 3; r++) free(s->cache_res[b][r]);
    }
    free(s->cache_out);
    free(s);
}

/* snake(x, a) = x + sin(a*x)^2 / a as ggml_mul, ggml_sin, ggml_sqr, ggml_div,
 * ggml_add (src/audio_vae_v2.c:483-503). */
static inline float vo_snake(float x, float a) {
    const float t = x * a;
    const float st = sinf(t);
    const float sq = st * st;
    const float corr = sq / a;
    return x + corr;
}

static void snake_rows(float *x, int T, int C, const float *alpha) {
    if (!alpha) return;
    for (int t = 0; t < T; t++)
        for (int c = 0; c < C; c++) x[(size_t)t * C + c] = vo_snake(x[(size_t)t * C + c], alpha[c]);
}

/* History + input, the cache_prepend of src/audio_vae_stream.c:184-226; the
 * cache then keeps the last `L` rows of the combination (:216-225). */
static float *prepend(float *cache, int L, const float *x, int T, int C) {
    float *comb = (float *)malloc((size_t)(L + T) * C * sizeof(float));
    if (!comb) return NULL;
    memcpy(comb, cache, (size_t)L * C * sizeof(float));
    memcpy(comb + (size_t)L * C, x, (size_t)T * C * sizeof(float));
    memcpy(cache, comb + (size_t)T * C, (size_t)L * C * sizeof(float));
    return comb;
}

/* Causal depthwise conv, kernel 7, dilation d, over history+input
 * (depthwise_conv1d, src/audio_vae_v2.c:214-319): y = dot + bias.
 * w: [C][7] (ggml [7, 1, C]). */
static int depthwise7(float *cache, int d, const float *x, int T, int C, const float *w, const float *bias,
                      float *y) {
    const int L = 6 * d;
    float *comb = prepend(cache, L, x, T, C);
    if (!comb) return -1;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++)
        for (int c = 0; c < C; c++) {
            VO_ACC acc = 0;
            for (int j = 0; j < 7; j++) acc += (VO_ACC)w[(size_t)c * 7 + j] * (VO_ACC)comb[(size_t)(t + j * d) * C + c];
            float v = (float)acc;
            if (bias) v = v + bias[c];
            y[(size_t)t * C + c] = v;
        }
    free(comb);
    return 0;
}

/* Pointwise conv (kernel 1): y[t][o] = dot(W[o], x[t]) + bias[o]
 * (conv1d_layer with pad 0, :353-407).  w: [Co][Ci] (ggml [1, Ci, Co]).
 * With skip: y = skip + that (the residual add of :627-629). */
static void pointwise(const float *x, int T, int Ci, int Co, const float *w, const float *bias, const float *skip,
                      float *y) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++)
        for (int o = 0; o < Co; o++) {
            VO_ACC acc = 0;
            const float *wr = w + (size_t)o * Ci, *xr = x + (size_t)t * Ci;
            for (int i = 0; i < Ci; i++) acc += (VO_ACC)wr[i] * (VO_ACC)xr[i];
            float v = (float)acc;
            if (bias) v = v + bias[o];
            if (skip) v = skip[(size_t)t * Co + o] + v;
            y[(size_t)t * Co + o] = v;
        }
}

/* Streaming transposed conv, kernel 2s, stride s (stream_upconv,
 * src/audio_vae_stream.c:256-277 over vcpm_vae_upconv_transpose1d): output
 * time q*s + r takes input q-1 (the cache for q = 0) through tap s + r,
 * then input q through tap r, added in that order into a zeroed
 * accumulator, then the bias.  w: [Ci][Co][2s] (ggml [2s, Co, Ci]). */
static int upconv(float *cache, const float *x, int T, int Ci, int Co, int s, const float *w, const float *bias,
                  float *y) {
    float *comb = prepend(cache, 1, x, T, Ci);
    if (!comb) return -1;
    const int K = 2 * s;
    int rc = 0;
    /* per output row q: accumulators [s][Co] for both taps, filled with the
     * weight rows in memory order (input channel ascending, so each sum has
     * the same order as a per-output loop) */
#pragma omp parallel
    {
        VO_ACC *a0 = (VO_ACC *)malloc((size_t)s * Co * sizeof(VO_ACC));
        VO_ACC *a1 = (VO_ACC *)malloc((size_t)s * Co * sizeof(VO_ACC));
        if (!a0 || !a1) {
#pragma omp atomic write
            rc = -1;
        } else {
#pragma omp for schedule(static)
            for (int q = 0; q < T; q++) {
                const float *xp = comb + (size_t)q * Ci, *xc = comb + (size_t)(q + 1) * Ci;
                for (size_t k = 0; k < (size_t)s * Co; k++) a0[k] = a1[k] = 0;
                for (int i = 0; i < Ci; i++) {
                    const float *wi = w + (size_t)i * Co * K;
                    const VO_ACC vp = (VO_ACC)xp[i], vc = (VO_ACC)xc[i];
                    for (int o = 0; o < Co; o++)
                        for (int r = 0; r < s; r++) {
                            a0[(size_t)r * Co + o] += (VO_ACC)wi[(size_t)o * K + s + r] * vp;
                            a1[(size_t)r * Co + o] += (VO_ACC)wi[(size_t)o * K + r] * vc;
                        }
                }
                for (int r = 0; r < s; r++)
                    for (int o = 0; o < Co; o++) {
                        float v = 0.0f;
                        v = v + (float)a0[(size_t)r * Co + o];
                        v = v + (float)a1[(size_t)r * Co + o];
                        if (bias) v = v + bias[o];
                        y[((size_t)q * s + r) * Co + o] = v;
                    }
            }
        }
        free(a0);
        free(a1);
    }
    free(comb);
    return rc;
}

/* Output conv, kernel 7, C -> 1, over history+input (model.9 through
 * stream_conv, :554-560), then tanh (:561).  w: [C][7] (ggml [7, C, 1]),
 * summed in im2col order (channel-major, tap-minor). */
static int out_conv(float *cache, const float *x, int T, int C, const float *w, const float *bias, float *audio) {
    float *comb = prepend(cache, 6, x, T, C);
    if (!comb) return -1;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++) {
        VO_ACC acc = 0;
        for (int i = 0; i < C; i++)
            for (int j = 0; j < 7; j++) acc += (VO_ACC)w[(size_t)i * 7 + j] * (VO_ACC)comb[(size_t)(t + j) * C + i];
        float v = (float)acc;
        if (bias) v = v + bias[0];
        audio[t] = tanhf(v);
    }
    free(comb);
    return 0;
}

int vo_vae_stream_decode(vo_vae_stream *s, const float *latent, int n, float *audio) {
    if (!s || !latent || !audio || n <= 0) return -1;
    const vo_vae_config *c = &s->cfg;
    const float *const *w = s->w;
    size_t mx = (size_t)n * c->decoder_dim;
    {
        int T = n;
        for (int b = 0; b < 6; b++) {
            T *= c->rates[b];
            const size_t v = (size_t)T * vo_vae_channels(c, b + 1);
            if (v > mx) mx = v;
        }
    }
    float *h = (float *)malloc(mx * sizeof(float));
    float *t1 = (float *)malloc(mx * sizeof(float));
    float *t2 = (float *)malloc(mx * sizeof(float));
    float *x0 = (float *)malloc((size_t)n * c->latent_dim * sizeof(float));
    int rc = (h && t1 && t2 && x0) ? 0 : -1;
    if (!rc) {
        /* model.0: depthwise k7 over the latent; model.1: pointwise to D */
        rc = depthwise7(s->cache_in, 1, latent, n, c->latent_dim, w[VO_VAE_IN_DW_W], w[VO_VAE_IN_DW_B], x0);
        if (!rc) pointwise(x0, n, c->latent_dim, c->decoder_dim, w[VO_VAE_IN_PW_W], w[VO_VAE_IN_PW_B], NULL, h);
    }
    int T = n;
    for (int b = 0; b < 6 && !rc; b++) {
        const int ci = vo_vae_channels(c, b), co = vo_vae_channels(c, b + 1), st = c->rates[b];
        const int base = VO_VAE_BLOCK0 + b * VO_VAE_BLOCK_SLOTS;
        /* sr_cond scale/bias (src/audio_vae_stream.c:468-496): ggml_mul then ggml_add */
        const float *sc = w[base + VO_VAE_B_SR_SCALE], *sb = w[base + VO_VAE_B_SR_BIAS];
        if (sc && sb)
            for (int t = 0; t < T; t++)
                for (int k = 0; k < ci; k++) {
                    float v = h[(size_t)t * ci + k] * sc[k];
                    h[(size_t)t * ci + k] = v + sb[k];
                }
        snake_rows(h, T, ci, w[base + VO_VAE_B_ALPHA]);
        rc = upconv(s->cache_up[b], h, T, ci, co, st, w[base + VO_VAE_B_UP_W], w[base + VO_VAE_B_UP_B], t1);
        if (rc) break;
        T *= st;
        memcpy(h, t1, (size_t)T * co * sizeof(float));
        for (int r = 0; r < 3 && !rc; r++) {
            const int rb = base + VO_VAE_B_RES0 + r * VO_VAE_RES_SLOTS;
            memcpy(t1, h, (size_t)T * co * sizeof(float));
            snake_rows(t1, T, co, w[rb + VO_VAE_R_ALPHA0]);
            rc = depthwise7(s->cache_res[b][r], vo_vae_dil[r], t1, T, co, w[rb + VO_VAE_R_DW_W], w[rb + VO_VAE_R_DW_B],
                            t2);
            if (rc) break;
            snake_rows(t2, T, co, w[rb + VO_VAE_R_ALPHA2]);
            pointwise(t2, T, co, co, w[rb + VO_VAE_R_PW_W], w[rb + VO_VAE_R_PW_B], h, t1);
            memcpy(h, t1, (size_t)T * co * sizeof(float));
        }
    }
    if (!rc) {
        const int cl = vo_vae_channels(c, 6);
        snake_rows(h, T, cl, w[VO_VAE_OUT_ALPHA]);
        rc = out_conv(s->cache_out, h, T, cl, w[VO_VAE_OUT_W], w[VO_VAE_OUT_B], audio);
    }
    free(h);
    free(t1);
    free(t2);
    free(x0);
    return rc;
}

int vo_vae_decode(const vo_vae_config *cfg, const float *const *w, const float *latent, int n, float *audio) {
    vo_vae_stream *s = vo_vae_stream_create(cfg, w);
    if (!s) return -1;
    const int rc = vo_vae_stream_decode(s, latent, n, audio);
    vo_vae_stream_free(s);
    return rc;
}
