/* vcpm_gen_run.c -- a C11 host driver of libvcpm_b200.so, written against
 * include/vcpm_b200.h alone (no CUDA headers, no C++).
 *
 * It replays the reference's generation loop (src/gen_run.c:60-241) for a
 * batch of utterances with a small synthetic model: prompt embeddings ->
 * vb_gen_prefill, then per patch vb_gen_step_stop (mu -> CFM -> LocEnc ->
 * TSLM -> FSQ -> RALM -> stop predictor with the min-length gate), the
 * latent patch of every utterance through the streaming AudioVAE decoder,
 * and the reference's per-utterance break (:195-213): utterances whose stop
 * flag is set are retired from the generator and the VAE streams alike
 * (vb_gen_retire / vb_vae_stream_retire compact both batches), the rest go
 * on until max_len patches.
 *
 *   vcpm_gen_run layout
 *       prints sizeof / offsetof of the public structs as one JSON object
 *       (no device needed; the Python binding's ctypes layouts are checked
 *       against it)
 *   vcpm_gen_run run [batch] [max_len] [min_len] [seed]
 *       builds the synthetic model on device 0, generates, prints one JSON
 *       line (patches per utterance, an audio checksum, device status) and
 *       exits 0 on success, 1 on any library error (its message on stderr).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "vcpm_b200.h"

/* ------------------------------------------------------------ layout */
#define FIELD(T, f) printf("\"%s.%s\": %zu, ", #T, #f, offsetof(T, f))
#define SIZE(T) printf("\"%s\": %zu, ", #T, sizeof(T))

static void print_layout(void) {
    printf("{");
    SIZE(vb_lm_config);
    FIELD(vb_lm_config, eps);
    FIELD(vb_lm_config, rope_theta);
    FIELD(vb_lm_config, no_rope);
    FIELD(vb_lm_config, scale_depth);
    FIELD(vb_lm_config, wtype);
    SIZE(vb_layer_host);
    FIELD(vb_layer_host, down);
    FIELD(vb_layer_host, attn_norm);
    FIELD(vb_layer_host, ffn_norm);
    SIZE(vb_dit_config);
    FIELD(vb_dit_config, feat_dim);
    FIELD(vb_dit_config, patch);
    FIELD(vb_dit_config, eps);
    FIELD(vb_dit_config, wtype);
    SIZE(vb_dit_host);
    FIELD(vb_dit_host, t_w1);
    FIELD(vb_dit_host, norm);
    FIELD(vb_dit_host, layers);
    SIZE(vb_gemv_op);
    FIELD(vb_gemv_op, ldx);
    FIELD(vb_gemv_op, y);
    FIELD(vb_gemv_op, bias);
    FIELD(vb_gemv_op, flags);
    FIELD(vb_gemv_op, M);
    FIELD(vb_gemv_op, group);
    FIELD(vb_gemv_op, wait_group);
    SIZE(vb_gen_parts);
    FIELD(vb_gen_parts, dit);
    FIELD(vb_gen_parts, stop_head);
    FIELD(vb_gen_parts, enc_in_bias);
    FIELD(vb_gen_parts, stop_head_bias);
    FIELD(vb_gen_parts, feat_dim);
    FIELD(vb_gen_parts, patch);
    FIELD(vb_gen_parts, fsq_scale);
    FIELD(vb_gen_parts, eps);
    FIELD(vb_gen_parts, cfm_steps);
    FIELD(vb_gen_parts, cfg_value);
    SIZE(vb_vae_config);
    FIELD(vb_vae_config, decoder_dim);
    FIELD(vb_vae_config, rates);
    FIELD(vb_vae_config, weight_type);
    printf("\"VB_VAE_N_SLOTS\": %d}\n", (int)VB_VAE_N_SLOTS);
}

/* ------------------------------------------------- synthetic weights */
static uint64_t rng_state = 0x9E3779B97F4A7C15ull;

static uint64_t rng_next(void) { /* xorshift64* */
    rng_state ^= rng_state >> 12;
    rng_state ^= rng_state << 25;
    rng_state ^= rng_state >> 27;
    return rng_state * 0x2545F4914F6CDD1Dull;
}

static float rng_uniform(void) { return (float)((rng_next() >> 40) * (1.0 / 16777216.0)); } /* [0, 1) */

static float rng_normal(void) { /* sum of four uniforms, unit variance */
    float s = 0.0f;
    for (int i = 0; i < 4; i++) s += rng_uniform();
    return (s - 2.0f) * 1.7320508f;
}

/* IEEE binary16 bits of a float, round to nearest even (normal range and
 * gradual underflow; values here are small and finite). */
static uint16_t half_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t m = x & 0x7fffffu;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* Q8_0 weight [N][K] in GGUF block storage (fp16 scale + 32 int8 per
 * block), entries ~ N(0, std^2). */
static void *q8_weight(int64_t N, int64_t K, float std) {
    const int64_t nb = N * (K / 32);
    uint8_t *b = (uint8_t *)malloc((size_t)nb * 34);
    if (!b) return NULL;
    for (int64_t i = 0; i < nb; i++) {
        const uint16_t d = half_bits(std * 2.5f / 127.0f);
        memcpy(b + i * 34, &d, 2);
        for (int j = 0; j < 32; j++) {
            float q = rng_normal() * 127.0f / 2.5f;
            if (q > 127.0f) q = 127.0f;
            if (q < -127.0f) q = -127.0f;
            b[i * 34 + 2 + j] = (uint8_t)(int8_t)lrintf(q);
        }
    }
    return b;
}

static float *f32_vec(int64_t n, float mean, float std) {
    float *v = (float *)malloc((size_t)n * 4);
    if (!v) return NULL;
    for (int64_t i = 0; i < n; i++) v[i] = mean + std * rng_normal();
    return v;
}

/* every host allocation, freed at exit */
static void *owned[4096];
static int n_owned = 0;

static void *keep(void *p) {
    if (!p) {
        fprintf(stderr, "host allocation failed\n");
        exit(1);
    }
    if (n_owned < (int)(sizeof(owned) / sizeof(owned[0]))) owned[n_owned++] = p;
    return p;
}

static vb_ctx *ctx = NULL;

static void check(int rc, const char *what) {
    if (rc != VB_OK) {
        fprintf(stderr, "%s failed (%d): %s\n", what, rc, ctx ? vb_last_error(ctx) : "");
        exit(1);
    }
}

/* model shape: a scaled-down VoxCPM (same structure as the real one) */
enum { H = 256, NH = 4, NKV = 2, HD = 64, FFN = 512, TSLM_L = 2, RALM_L = 2, DH = 256, DFFN = 512,
       DIT_L = 2, ENC_L = 2, FEAT = 64, PATCH = 4, FSQ = 64, PROMPT = 24 };

static void layer(vb_layer_host *L, int hidden, int ffn) {
    L->q = keep(q8_weight(NH * HD, hidden, 0.05f));
    L->k = keep(q8_weight(NKV * HD, hidden, 0.05f));
    L->v = keep(q8_weight(NKV * HD, hidden, 0.05f));
    L->o = keep(q8_weight(hidden, NH * HD, 0.05f));
    L->gate = keep(q8_weight(ffn, hidden, 0.05f));
    L->up = keep(q8_weight(ffn, hidden, 0.05f));
    L->down = keep(q8_weight(hidden, ffn, 0.05f));
    L->attn_norm = keep(f32_vec(hidden, 1.0f, 0.02f));
    L->ffn_norm = keep(f32_vec(hidden, 1.0f, 0.02f));
}

static vb_weight reg_q8(int64_t K, int64_t N, float std) {
    void *b = keep(q8_weight(N, K, std));
    vb_weight w = NULL;
    check(vb_weight_register(ctx, VB_TYPE_Q8_0, K, N, b, (size_t)(N * (K / 32) * 34), &w), "vb_weight_register");
    return w;
}

static float *dev_vec(int64_t n, float mean, float std) {
    float *h = (float *)keep(f32_vec(n, mean, std));
    void *d = NULL;
    check(vb_malloc(ctx, (size_t)n * 4, &d), "vb_malloc");
    check(vb_memcpy_h2d(ctx, d, h, (size_t)n * 4), "vb_memcpy_h2d");
    return (float *)d;
}

static const void *vae_tensor(int slot, const int *rates) {
    const int D = 256, LAT = FEAT;
    if (slot == VB_VAE_IN_DW_W) return keep(f32_vec(LAT * 7, 0.0f, 0.38f));
    if (slot == VB_VAE_IN_DW_B) return keep(f32_vec(LAT, 0.0f, 0.02f));
    if (slot == VB_VAE_IN_PW_W) return keep(f32_vec((int64_t)D * LAT, 0.0f, 0.125f));
    if (slot == VB_VAE_IN_PW_B) return keep(f32_vec(D, 0.0f, 0.02f));
    if (slot == VB_VAE_OUT_ALPHA) return keep(f32_vec(D >> 6, 1.0f, 0.2f));
    if (slot == VB_VAE_OUT_W) return keep(f32_vec((D >> 6) * 7, 0.0f, 0.03f));
    if (slot == VB_VAE_OUT_B) return keep(f32_vec(1, 0.0f, 0.02f));
    const int b = (slot - VB_VAE_BLOCK0) / VB_VAE_BLOCK_SLOTS, r = (slot - VB_VAE_BLOCK0) % VB_VAE_BLOCK_SLOTS;
    const int ci = D >> b, co = D >> (b + 1);
    if (r == VB_VAE_B_SR_SCALE || r == VB_VAE_B_SR_BIAS) return NULL;
    if (r == VB_VAE_B_ALPHA) return keep(f32_vec(ci, 1.0f, 0.2f));
    if (r == VB_VAE_B_UP_W) return keep(f32_vec((int64_t)ci * co * 2 * rates[b], 0.0f, 1.0f / sqrtf(2.0f * ci)));
    if (r == VB_VAE_B_UP_B) return keep(f32_vec(co, 0.0f, 0.02f));
    const int ur = (r - VB_VAE_B_RES0) % VB_VAE_RES_SLOTS;
    if (ur == VB_VAE_R_ALPHA0 || ur == VB_VAE_R_ALPHA2) return keep(f32_vec(co, 1.0f, 0.2f));
    if (ur == VB_VAE_R_DW_W) return keep(f32_vec(co * 7, 0.0f, 0.38f));
    if (ur == VB_VAE_R_PW_W) return keep(f32_vec((int64_t)co * co, 0.0f, 1.0f / sqrtf(4.0f * co)));
    return keep(f32_vec(co, 0.0f, 0.02f)); /* R_DW_B, R_PW_B */
}

static int run(int B, int max_len, int min_len, uint64_t seed) {
    int ndev = 0;
    check(vb_device_count(&ndev), "vb_device_count");
    if (ndev < 1) {
        fprintf(stderr, "no device\n");
        return 1;
    }
    check(vb_create(0, &ctx), "vb_create");
    rng_state ^= seed * 0x9E3779B97F4A7C15ull;

    /* stacks */
    vb_layer_host tl[TSLM_L], rl[RALM_L], el[ENC_L], dl[DIT_L];
    for (int i = 0; i < TSLM_L; i++) layer(&tl[i], H, FFN);
    for (int i = 0; i < RALM_L; i++) layer(&rl[i], H, FFN);
    for (int i = 0; i < ENC_L; i++) layer(&el[i], DH, DFFN);
    for (int i = 0; i < DIT_L; i++) layer(&dl[i], DH, DFFN);
    const vb_lm_config tcfg = {H, NH, NKV, HD, FFN, TSLM_L, 1e-5f, 10000.0f, 0, 0.0f, VB_TYPE_Q8_0};
    const vb_lm_config rcfg = {H, NH, NKV, HD, FFN, RALM_L, 1e-5f, 10000.0f, 1, 0.0f, VB_TYPE_Q8_0};
    const vb_lm_config ecfg = {DH, NH, NKV, HD, DFFN, ENC_L, 1e-5f, 10000.0f, 0, 0.0f, VB_TYPE_Q8_0};
    vb_lm *tslm = NULL, *ralm = NULL, *enc = NULL;
    check(vb_lm_create(ctx, &tcfg, tl, (const float *)keep(f32_vec(H, 1.0f, 0.02f)), &tslm), "vb_lm_create tslm");
    check(vb_lm_create(ctx, &rcfg, rl, (const float *)keep(f32_vec(H, 1.0f, 0.02f)), &ralm), "vb_lm_create ralm");
    check(vb_lm_create(ctx, &ecfg, el, NULL, &enc), "vb_lm_create enc");

    const vb_dit_config dcfg = {DH, DIT_L, NH, NKV, DFFN, HD, FEAT, PATCH, 1e-5f, VB_TYPE_Q8_0};
    vb_dit_host dh;
    dh.in_proj = keep(q8_weight(DH, FEAT, 0.1f));
    dh.cond_proj = keep(q8_weight(DH, FEAT, 0.1f));
    dh.out_proj = keep(q8_weight(FEAT, DH, 0.05f));
    dh.in_bias = keep(f32_vec(DH, 0.0f, 0.02f));
    dh.cond_bias = keep(f32_vec(DH, 0.0f, 0.02f));
    dh.out_bias = keep(f32_vec(FEAT, 0.0f, 0.02f));
    dh.t_w1 = keep(q8_weight(DH, DH, 0.05f));
    dh.t_w2 = keep(q8_weight(DH, DH, 0.05f));
    dh.dt_w1 = keep(q8_weight(DH, DH, 0.05f));
    dh.dt_w2 = keep(q8_weight(DH, DH, 0.05f));
    dh.t_b1 = keep(f32_vec(DH, 0.0f, 0.02f));
    dh.t_b2 = keep(f32_vec(DH, 0.0f, 0.02f));
    dh.dt_b1 = keep(f32_vec(DH, 0.0f, 0.02f));
    dh.dt_b2 = keep(f32_vec(DH, 0.0f, 0.02f));
    dh.norm = keep(f32_vec(DH, 1.0f, 0.02f));
    dh.layers = dl;
    vb_dit *dit = NULL;
    check(vb_dit_create(ctx, &dcfg, &dh, &dit), "vb_dit_create");

    /* projections and the stop predictor */
    vb_gen_parts p;
    memset(&p, 0, sizeof(p));
    p.tslm = tslm;
    p.ralm = ralm;
    p.enc = enc;
    p.dit = dit;
    p.enc_in = reg_q8(FEAT, DH, 0.1f);
    p.enc_to_lm = reg_q8(DH, H, 0.05f);
    p.lm_to_dit = reg_q8(H, DH, 0.05f);
    p.res_to_dit = reg_q8(H, DH, 0.05f);
    p.fsq_in = reg_q8(H, FSQ, 0.05f);
    p.fsq_out = reg_q8(FSQ, H, 0.05f);
    p.fusion = reg_q8(2 * H, H, 0.05f);
    p.stop_proj = reg_q8(H, H, 0.05f);
    p.stop_head = reg_q8(H, 2, 0.2f);
    p.enc_in_bias = dev_vec(DH, 0.0f, 0.02f);
    p.enc_special = dev_vec(DH, 0.0f, 0.5f);
    p.enc_norm = dev_vec(DH, 1.0f, 0.02f);
    p.enc_to_lm_bias = dev_vec(H, 0.0f, 0.02f);
    p.lm_to_dit_bias = dev_vec(DH, 0.0f, 0.02f);
    p.res_to_dit_bias = dev_vec(DH, 0.0f, 0.02f);
    p.fsq_in_bias = dev_vec(FSQ, 0.0f, 0.02f);
    p.fsq_out_bias = dev_vec(H, 0.0f, 0.02f);
    p.fusion_bias = dev_vec(H, 0.0f, 0.02f);
    p.stop_proj_bias = dev_vec(H, 0.0f, 0.02f);
    p.stop_head_bias = NULL;
    p.feat_dim = FEAT;
    p.patch = PATCH;
    p.fsq_scale = 9.0f;
    p.eps = 1e-5f;
    p.cfm_steps = 10;
    p.cfg_value = 2.0f;

    /* AudioVAE V2 decoder, 4 channels after six x2 stages */
    const vb_vae_config vcfg = {FEAT, 256, {2, 2, 2, 2, 2, 2}, VB_TYPE_F32};
    const void *vt[VB_VAE_N_SLOTS];
    for (int s = 0; s < VB_VAE_N_SLOTS; s++) vt[s] = vae_tensor(s, vcfg.rates);
    vb_vae vae = NULL;
    vb_vae_stream vst = NULL;
    check(vb_vae_create(ctx, &vcfg, vt, &vae), "vb_vae_create");
    check(vb_vae_stream_create(ctx, vae, B, PATCH, &vst), "vb_vae_stream_create");
    const int spp = vb_vae_stream_patch_samples(vst);

    /* the loop of src/gen_run.c:166-215 */
    vb_gen g = NULL;
    check(vb_gen_create(ctx, &p, B, PROMPT + max_len + 2, &g), "vb_gen_create");
    check(vb_gen_set_min_len(g, min_len), "vb_gen_set_min_len");
    float *emb = dev_vec((int64_t)B * PROMPT * H, 0.0f, 0.5f);
    check(vb_gen_prefill(ctx, g, PROMPT, emb), "vb_gen_prefill");
    void *patches = NULL, *audio = NULL, *stop_d = NULL;
    const size_t prow = (size_t)PATCH * FEAT * 4;
    check(vb_malloc(ctx, (size_t)B * prow, &patches), "vb_malloc");
    check(vb_malloc(ctx, (size_t)B * spp * 4, &audio), "vb_malloc");
    check(vb_malloc(ctx, (size_t)B * 4, &stop_d), "vb_malloc");
    int32_t *active = (int32_t *)keep(calloc((size_t)B, 4)), *stop = (int32_t *)keep(calloc((size_t)B, 4));
    int32_t *done = (int32_t *)keep(calloc((size_t)B, 4));
    int *n_patches = (int *)keep(calloc((size_t)B, sizeof(int)));
    float *pcm = (float *)keep(malloc((size_t)B * spp * 4));
    double checksum = 0.0;
    int steps = 0;
    for (int step = 0; step < max_len; step++) {
        const int n = vb_gen_active(g, active);
        if (n <= 0) break;
        check(vb_gen_step_stop(ctx, g, seed, (float *)patches, NULL, (int32_t *)stop_d), "vb_gen_step_stop");
        /* the VAE streams are retired with the generator's rows, so the
         * patches' row order is the streams' */
        check(vb_vae_stream_decode(ctx, vst, (const float *)patches, PATCH, (float *)audio), "vb_vae_stream_decode");
        check(vb_memcpy_d2h(ctx, pcm, audio, (size_t)n * spp * 4), "vb_memcpy_d2h");
        check(vb_memcpy_d2h(ctx, stop, stop_d, (size_t)n * 4), "vb_memcpy_d2h");
        check(vb_sync(ctx), "vb_sync");
        int n_done = 0;
        for (int j = 0; j < n; j++) {
            const int u = active[j];
            n_patches[u]++;
            for (int s = 0; s < spp; s++) checksum += fabs((double)pcm[(size_t)j * spp + s]);
            if (stop[j]) done[n_done++] = u;
        }
        if (n_done) {
            check(vb_gen_retire(ctx, g, n_done, done), "vb_gen_retire");
            check(vb_vae_stream_retire(ctx, vst, n_done, done), "vb_vae_stream_retire");
        }
        steps++;
    }
    int derr = 0;
    check(vb_device_status(ctx, &derr), "vb_device_status");
    printf("{\"batch\": %d, \"max_len\": %d, \"min_len\": %d, \"steps\": %d, \"samples_per_patch\": %d, "
           "\"patches\": [", B, max_len, min_len, steps, spp);
    for (int u = 0; u < B; u++) printf("%s%d", u ? ", " : "", n_patches[u]);
    printf("], \"audio_abs_sum\": %.6f, \"finite\": %s, \"device_error\": %d}\n", checksum,
           isfinite(checksum) ? "true" : "false", derr);

    vb_gen_destroy(ctx, g);
    vb_vae_stream_destroy(ctx, vst);
    vb_vae_destroy(ctx, vae);
    vb_weight ws[] = {p.enc_in, p.enc_to_lm, p.lm_to_dit, p.res_to_dit, p.fsq_in, p.fsq_out, p.fusion, p.stop_proj,
                      p.stop_head};
    for (size_t i = 0; i < sizeof(ws) / sizeof(ws[0]); i++) vb_weight_release(ctx, ws[i]);
    vb_dit_destroy(ctx, dit);
    vb_lm_destroy(ctx, enc);
    vb_lm_destroy(ctx, ralm);
    vb_lm_destroy(ctx, tslm);
    vb_destroy(ctx);
    ctx = NULL;
    return derr == 0 && isfinite(checksum) ? 0 : 1;
}

int main(int argc, char **argv) {
    if (argc >= 2 && strcmp(argv[1], "layout") == 0) {
        print_layout();
        return 0;
    }
    if (argc >= 2 && strcmp(argv[1], "run") == 0) {
        const int B = argc > 2 ? atoi(argv[2]) : 4;
        const int max_len = argc > 3 ? atoi(argv[3]) : 12;
        const int min_len = argc > 4 ? atoi(argv[4]) : 2;
        const uint64_t seed = argc > 5 ? strtoull(argv[5], NULL, 10) : 1234u;
        if (B < 1 || B > 8 || max_len < 1) {
            fprintf(stderr, "batch 1..8, max_len >= 1\n");
            return 2;
        }
        const int rc = run(B, max_len, min_len, seed);
        for (int i = 0; i < n_owned; i++) free(owned[i]);
        return rc;
    }
    fprintf(stderr, "usage: %s layout | run [batch] [max_len] [min_len] [seed]\n", argv[0]);
    return 2;
}
