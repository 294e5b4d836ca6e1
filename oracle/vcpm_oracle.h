/*
 * vcpm_oracle.h -- CPU restatement of VoxCPM-C's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 kernels in voxcpm-cpp_b200/.  Only tests/, __graft_entry__.smoke()
 * and the CPU-baseline legs of bench.py may load it; the product path never
 * links it and never falls back to it.
 *
 * What it restates (reference paths are relative to the voxcpm-cpp tree):
 *   - ggml-CPU semantics of the ops the reference graphs use: Q8_0 weight and
 *     activation quantization, Q8_0/F16/F32 mat-mul with fp32 results,
 *     rms_norm, NEOX rope_ext with freq_factors, soft_max, silu, tanh/round
 *     and the F32->BF16->F32 cast.  ggml v0.15.2 is a third-party dependency
 *     fetched at configure time (CMakeLists.txt:55-68) and is not in the tree;
 *     its behaviour is restated from its documented algorithms.
 *   - the graph builders of the reference: src/minicpm4.c (norm, rope,
 *     attention, mlp, block, forward), src/locdit.c (LocDiT estimator),
 *     src/locenc.c (feature encoder), src/fsq.c, src/cfm_solver.c, the
 *     CFM/LM-update loop of src/gen_step.c and the stop predictor of
 *     src/gen_stop.c.
 *
 * Parity status: the CFM schedule/CFG-Zero* goldens, the op fixtures and
 * the small known-answer tests of the reference pin the non-quantized ops.
 * Q8_0 activation quantization and the Q8_0 mat-mul are NOT pinned by any
 * reference test (every reference fixture uses F32 weights); the weight
 * quantizer is cross-checked bit-for-bit against gguf-py's Q8_0 quantizer.
 *
 * Layout conventions (ggml, src/minicpm4.c:5-8): a weight W with ggml shape
 * [K, N] is N rows of K contiguous elements.  Activations are row-major
 * [M][K] (one token per row); mat-mul results are [M][N].
 */
#ifndef VCPM_ORACLE_H
#define VCPM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type enum values for the weight types on the path. */
enum { VO_TYPE_F32 = 0, VO_TYPE_F16 = 1, VO_TYPE_Q8_0 = 8 };

/* Activation-quantization rounding rule.
 *   VO_QRULE_X86: ggml-CPU x86 SIMD rule: d = amax/127, id = 127/amax,
 *                 q = round-half-even(x*id).
 *   VO_QRULE_REF: ggml reference rule (weights, tools/quantize.c:292):
 *                 d = amax/127, id = 1/d, q = round-half-away(x*id). */
enum { VO_QRULE_X86 = 0, VO_QRULE_REF = 1 };

#define VO_QK8_0 32
#define VO_Q8_0_BYTES 34

/* ---- scalar conversions ---- */
uint16_t vo_fp32_to_bf16(float x);
float    vo_bf16_to_fp32(uint16_t h);
float    vo_bf16_round(float x);
uint16_t vo_fp32_to_fp16(float x);
float    vo_fp16_to_fp32(uint16_t h);
void     vo_bf16_round_array(float *x, int64_t n);

/* ---- Q8_0 ---- */
void vo_quantize_q8_0(const float *x, void *blocks, int64_t n, int rule);
void vo_dequantize_q8_0(const void *blocks, float *y, int64_t n);
size_t vo_row_bytes(int type, int64_t K);
int vo_get_rows(int type, const void *table, int64_t K, int64_t n_rows, const int32_t *ids, int64_t n,
                float *out);

/* y[m*N+n] = sum_k W[n,k]*x[m*K+k] with ggml-CPU operand conversion:
 * Q8_0 weights quantize x rows to Q8_0 (rule), F16 weights round x to fp16,
 * F32 weights use x as is.  Returns 0, or -1 on a bad argument. */
int vo_matmul(int wtype, const void *W, int64_t K, int64_t N,
              const float *x, int64_t M, float *y, int qrule, int nthreads);

/* ---- elementwise ops ---- */
void vo_rms_norm(const float *x, float *y, int64_t n, int64_t rows, float eps);
void vo_rms_norm_bf16(const float *x, const float *w, float *y, int64_t n,
                      int64_t rows, float eps);
float vo_silu(float x);
void vo_fsq_quantize(float *x, int64_t n, float quant_scale);
void vo_rope_cache(float *cs, int32_t pos, int head_dim, float theta,
                   const float *freq_factors);
void vo_rope_neox(float *x, int head_dim, int n_heads, int n_tokens,
                  int32_t pos0, float theta, const float *freq_factors);
const float *vo_longrope_short_factors(void);

/* ---- transformer (src/minicpm4.c) ---- */
typedef struct {
    int wtype;
    const void *q, *k, *v, *o, *gate, *up, *down;
    const float *attn_norm, *ffn_norm;
} vo_layer_weights;

typedef struct {
    int hidden, n_heads, n_kv_heads, head_dim, ffn, n_layers;
    float eps;
    float rope_theta;
    int no_rope;
    float scale_depth;
} vo_lm_config;

/* KV cache for one layer: F32 holding bf16 values, layout [cap][n_kv][hd]
 * (ggml [head_dim, n_kv_heads, capacity], src/minicpm4.c:106-116). */
typedef struct {
    float *k;
    float *v;
    int capacity;
    int n_used;
} vo_kv_layer;

typedef struct {
    int qrule;
    int nthreads;
    int bf16;         /* 1 = model semantics (bf16 casts), 0 = raw ops */
} vo_opts;

int vo_attention(const vo_lm_config *cfg, const vo_layer_weights *w,
                 vo_kv_layer *cache, const float *x, int T, int pos,
                 int no_causal, float *out, const vo_opts *o);
int vo_mlp(int wtype, const void *gate, const void *up, const void *down,
           int hidden, int ffn, const float *x, int T, float *out,
           const vo_opts *o);
int vo_block(const vo_lm_config *cfg, const vo_layer_weights *w,
             vo_kv_layer *cache, float *h, int T, int pos, int no_causal,
             float scale, const vo_opts *o);
int vo_lm_forward(const vo_lm_config *cfg, const vo_layer_weights *layers,
                  const float *final_norm, vo_kv_layer *caches,
                  const float *x, int T, int pos, float *out,
                  const vo_opts *o);

/* ---- LocDiT estimator (src/locdit.c) ---- */
typedef struct {
    int hidden, n_layers, n_heads, n_kv_heads, ffn, head_dim;
    int feat_dim, patch;
    float eps;
} vo_dit_config;

typedef struct {
    int wtype;
    const void *in_proj, *cond_proj, *out_proj;
    const float *in_bias, *cond_bias, *out_bias;
    const void *t_w1, *t_w2, *dt_w1, *dt_w2;
    const float *t_b1, *t_b2, *dt_b1, *dt_b2;
    const float *norm;
    const vo_layer_weights *layers;
} vo_dit_weights;

void vo_dit_time_sin(float t, int dim, float *out);
int vo_dit_forward(const vo_dit_config *cfg, const vo_dit_weights *w,
                   const float *x, const float *cond, float t, float dt,
                   const float *mu, float *out, const vo_opts *o);

/* ---- LocEnc feature encoder (src/locenc.c) ---- */
typedef struct {
    int hidden, n_layers, n_heads, n_kv_heads, ffn, head_dim, feat_dim;
    float eps;
} vo_enc_config;

typedef struct {
    int wtype;
    const void *in_proj;
    const float *in_bias, *special, *norm;
    const vo_layer_weights *layers;
} vo_enc_weights;

int vo_enc_forward(const vo_enc_config *cfg, const vo_enc_weights *w,
                   const float *patch, int P, float *cls_out,
                   const vo_opts *o);

/* ---- CFM (src/cfm_solver.c, src/gen_step.c) ---- */
float vo_cfm_sway_t_bf16(int step, int n_steps);
float vo_cfg_zero_star(float *negative, const float *positive, int n,
                       float cfg_value);
int vo_cfm_zero_star_steps(int n_steps);
void vo_cfm_noise(uint64_t seed, int ar_step, float *x, int n);
int vo_cfm_solve(const vo_dit_config *cfg, const vo_dit_weights *w,
                 const float *mu, const float *cond, float *x, int n_steps,
                 float cfg_value, const vo_opts *o);

/* ---- stop predictor (src/gen_stop.c:85-230) ---- */
/* stop_proj: hs*hs values read as W[j*hs + i] (input j, output i), any of
 * F32/F16/Q8_0 storage; proj_bias: F32 [hs] or NULL; stop_head: hs*2 values
 * read as H[2*j + o].  Writes the two logits; returns the argmax class
 * (class 0 wins ties) or -1. */
int vo_stop_predict(int proj_type, const void *proj_w, const float *proj_bias,
                    int head_type, const void *head_w, const float *hidden,
                    int hs, float *logits);

/* ---- misc host helpers (src/gen_init.c) ---- */
int vo_round_cache_capacity(int required, int model_max);

/* ---- deterministic synthetic data ---- */
void vo_fill_normal(uint64_t seed, float mean, float stddev, float *x,
                    int64_t n);

/* ---- AudioVAE V2 decoder (vcpm_oracle_vae.c) ------------------------- */
/* Decoder geometry: latent channels, decoder_dim D (block b maps D>>b to
 * D>>(b+1) channels, src/audio_vae_v2.c:40-43) and the six upsampling
 * strides (transposed-conv kernel 2*stride). */
typedef struct vo_vae_config {
    int latent_dim;
    int decoder_dim;
    int rates[6];
} vo_vae_config;

/* Tensor slots of the decoder, all F32 in GGUF element order; biases,
 * Snake alphas and sr_cond vectors are per channel.  Slot names follow
 * audio_vae.decoder.* in src/audio_vae_stream.c:362-561. */
enum {
    VO_VAE_IN_DW_W = 0,    /* model.0.weight.weight  [latent][7] depthwise  */
    VO_VAE_IN_DW_B = 1,    /* model.0.bias                                    */
    VO_VAE_IN_PW_W = 2,    /* model.1.weight.weight  [D][latent]             */
    VO_VAE_IN_PW_B = 3,    /* model.1.bias                                    */
    VO_VAE_BLOCK0 = 4,     /* first slot of model.2; model.(2+b) at BLOCK0 + b*BLOCK_SLOTS */
    VO_VAE_BLOCK_SLOTS = 23,
    VO_VAE_B_SR_SCALE = 0, /* sr_cond_model.(2+b) scale vector [Ci] or NULL   */
    VO_VAE_B_SR_BIAS = 1,  /* sr_cond_model.(2+b) bias vector  [Ci] or NULL   */
    VO_VAE_B_ALPHA = 2,    /* block.0.alpha [Ci]                              */
    VO_VAE_B_UP_W = 3,     /* block.1.weight.weight [Ci][Co][2*stride]        */
    VO_VAE_B_UP_B = 4,     /* block.1.bias [Co]                               */
    VO_VAE_B_RES0 = 5,     /* residual unit u (block.(2+u)) at B_RES0 + u*RES_SLOTS */
    VO_VAE_RES_SLOTS = 6,
    VO_VAE_R_ALPHA0 = 0,   /* block.0.alpha [Co]                              */
    VO_VAE_R_DW_W = 1,     /* block.1.weight.weight [Co][7] depthwise         */
    VO_VAE_R_DW_B = 2,
    VO_VAE_R_ALPHA2 = 3,   /* block.2.alpha [Co]                              */
    VO_VAE_R_PW_W = 4,     /* block.3.weight.weight [Co][Co]                  */
    VO_VAE_R_PW_B = 5,
    VO_VAE_OUT_ALPHA = 142, /* model.8.alpha [D>>6]                           */
    VO_VAE_OUT_W = 143,     /* model.9.weight.weight [D>>6][7]               */
    VO_VAE_OUT_B = 144,     /* model.9.bias [1]                               */
    VO_VAE_N_SLOTS = 145
};

typedef struct vo_vae_stream vo_vae_stream;
int vo_vae_check_config(const vo_vae_config *cfg);
int vo_vae_upsample(const vo_vae_config *cfg);
/* Streaming decoder state with zeroed history (vcpm_vae_stream_create);
 * `w` (VO_VAE_N_SLOTS pointers) must outlive it. */
vo_vae_stream *vo_vae_stream_create(const vo_vae_config *cfg, const float *const *w);
void vo_vae_stream_free(vo_vae_stream *s);
/* latent [n][latent_dim] time-major -> audio [n * upsample] in (-1, 1)
 * (vcpm_vae_stream_decode, src/audio_vae_stream.c:563-619). */
int vo_vae_stream_decode(vo_vae_stream *s, const float *latent, int n, float *audio);
/* Whole-utterance decode (vcpm_vae_v2_decode) = streaming from zero state. */
int vo_vae_decode(const vo_vae_config *cfg, const float *const *w, const float *latent, int n, float *audio);

#ifdef __cplusplus
}
#endif

#endif
