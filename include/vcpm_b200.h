/*
 * vcpm_b200.h -- C ABI of the B200 (sm_100a) quantized-weight hot path of
 * VoxCPM-C.
 *
 * This library replaces, for the Q8_0/F16 mat-muls and the attention glue
 * between them, the ggml dispatch of the reference runtime
 * (src/ggml_backend.c, src/ggml_backend.h:33-59) and the weight offload of
 * src/model_loader.c (vcpm_model_offload, src/model_loader.h:169).  The C11
 * host code and include/voxcpm.h of the reference stay unchanged; a
 * replacement src/ggml_backend.c routes matching graph nodes here.
 *
 * Conventions
 *   - Plain C types only; device buffers are passed as plain pointers that
 *     the caller obtained from vb_malloc (or any cudaMalloc'd memory of the
 *     context's device).
 *   - Return codes mirror vcpm_status (include/voxcpm.h:14-23): 0 OK,
 *     1 INVALID_ARG, 5 BACKEND, 6 OOM, 7 NOT_IMPLEMENTED.  Nothing aborts;
 *     vb_last_error() holds the message of the last failure.
 *   - One vb_ctx = one device + one CUDA stream, used by one host thread at a
 *     time; multi-GPU hosts create one context per device.  All work is
 *     enqueued asynchronously on the context stream; vb_sync() waits.
 *   - Weight shapes use ggml order: a weight of ggml shape [K, N] is N rows
 *     of K elements (src/minicpm4.c:5-8).  Activations are row-major [M][K]
 *     (one token per row) and mat-mul results [M][N], both fp32.
 */
#ifndef VCPM_B200_H
#define VCPM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (include/voxcpm.h:14-23). */
enum {
    VB_OK = 0,
    VB_ERR_INVALID_ARG = 1,
    VB_ERR_BACKEND = 5,
    VB_ERR_OOM = 6,
    VB_ERR_NOT_IMPLEMENTED = 7
};

/* Weight types: ggml type ids (GGML_TYPE_F32/F16/Q8_0). */
enum { VB_TYPE_F32 = 0, VB_TYPE_F16 = 1, VB_TYPE_Q8_0 = 8 };

/* Q8_0 activation rounding rule.  VB_QRULE_X86 is ggml-CPU's x86 SIMD rule
 * (id = 127/amax, round half to even), the default; VB_QRULE_REF is ggml's
 * reference rule (id = 1/d, round half away from zero). */
enum { VB_QRULE_X86 = 0, VB_QRULE_REF = 1 };

/* Output flags. */
#define VB_OUT_BF16 1u   /* round results F32->BF16->F32 (src/minicpm4.c:39-42) */

typedef struct vb_ctx vb_ctx;
typedef struct vb_weight_s *vb_weight;

/* ------------------------------------------------------------------ */
/* Context: replaces vcpm_backend_init / vcpm_backend_free            */
/* (src/ggml_backend.h:33-37).                                        */
/* ------------------------------------------------------------------ */
int vb_device_count(int *n);
int vb_create(int device, vb_ctx **out);
void vb_destroy(vb_ctx *ctx);
const char *vb_last_error(const vb_ctx *ctx);
/* Waits for all work on the context stream (the synchronous return of
 * vcpm_backend_compute_graph, src/ggml_backend.h:58-59). */
int vb_sync(vb_ctx *ctx);
/* Synchronise and report a device-side error code recorded by the
 * tensor-core mat-mul (0 = none; its waits are bounded, a timeout records a
 * code instead of hanging).  Returns VB_ERR_BACKEND when one was recorded. */
int vb_device_status(vb_ctx *ctx, int *device_error);
/* Use an external cudaStream_t (passed as void*); NULL restores the
 * context's own stream. */
int vb_set_stream(vb_ctx *ctx, void *cuda_stream);
void *vb_get_stream(vb_ctx *ctx);
/* Q8_0 activation rule for every later call on this context. */
int vb_set_qrule(vb_ctx *ctx, int rule);

/* CUDA-graph capture of a fixed sequence of calls on the context stream:
 * the device-side counterpart of the reference's persistent CFM graph
 * (src/gen_step.c:482-580), which builds a graph once and replays it.
 * Between begin and end only launches are recorded (no allocation, no
 * synchronisation); replay re-runs them on the same buffers. */
typedef struct vb_graph_s *vb_graph;
int vb_graph_begin(vb_ctx *ctx);
int vb_graph_end(vb_ctx *ctx, vb_graph *out);
int vb_graph_launch(vb_ctx *ctx, vb_graph g);
void vb_graph_destroy(vb_graph g);

/* CUDA events on the context stream, for timing replays from hosts that
 * do not link cudart: record, then elapsed milliseconds between two. */
typedef struct vb_event_s *vb_event;
int vb_event_create(vb_ctx *ctx, vb_event *out);
int vb_event_record(vb_ctx *ctx, vb_event e);
int vb_event_elapsed_ms(vb_event start, vb_event stop, float *ms);
void vb_event_destroy(vb_event e);

/* Device / pinned-host memory for hosts that do not link cudart. */
int vb_malloc(vb_ctx *ctx, size_t bytes, void **dptr);
int vb_free(vb_ctx *ctx, void *dptr);
int vb_host_alloc(vb_ctx *ctx, size_t bytes, void **hptr);
int vb_host_free(vb_ctx *ctx, void *hptr);
int vb_memcpy_h2d(vb_ctx *ctx, void *dst, const void *src, size_t bytes);
int vb_memcpy_d2h(vb_ctx *ctx, void *dst, const void *src, size_t bytes);
int vb_memcpy_d2d(vb_ctx *ctx, void *dst, const void *src, size_t bytes);
int vb_memset(vb_ctx *ctx, void *dst, int value, size_t bytes);

/* ------------------------------------------------------------------ */
/* Weights: replaces vcpm_model_offload (src/model_loader.h:169,      */
/* src/model_loader.c:615-700).  The GGUF bytes (34-byte Q8_0 blocks,  */
/* fp16 or fp32 rows) are uploaded and repacked once; the host buffer */
/* stays owned by the caller, the device copy by the context.         */
/* ------------------------------------------------------------------ */
int vb_weight_register(vb_ctx *ctx, int type, int64_t K, int64_t N,
                       const void *host, size_t nbytes, vb_weight *out);
int vb_weight_release(vb_ctx *ctx, vb_weight w);
int vb_weight_info(vb_weight w, int *type, int64_t *K, int64_t *N,
                   size_t *device_bytes);

/* ------------------------------------------------------------------ */
/* Ops on device pointers                                             */
/* ------------------------------------------------------------------ */

/* ggml_mul_mat(W, x) on a registered Q8_0/F16/F32 weight
 * (src/projections.h:24-29 and every call site of src/minicpm4.c,
 * src/locdit.c, src/gen_step.c): y[m][n] = sum_k W[n][k] x[m][k] with
 * ggml-CPU operand conversion (Q8_0: x quantized to Q8_0 per row; F16: x
 * rounded to fp16).  flags: VB_OUT_BF16.  Optional bias (F32 [N], device,
 * added before rounding, dit_add_bias_2d src/locdit.c:192-207). */
int vb_matmul(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, float *y,
              unsigned flags);
int vb_matmul_bias(vb_ctx *ctx, vb_weight w, const float *x, int64_t M,
                   const float *bias, float *y, unsigned flags);

/* Weight-streaming GEMV programs: a fixed list of ggml_mul_mat calls with
 * small M (the decode-time mat-muls of src/minicpm4.c:270-458, M = batch)
 * run by ONE persistent launch that streams every weight through shared
 * memory once (the B200 replacement for dispatching each mat-mul node of a
 * graph separately, src/ggml_backend.c:557-599).  Ops are grouped: ops of
 * one group run concurrently; an op with wait_group >= 0 reads its x only
 * after every op of that earlier group has finished on all SMs.  Groups are
 * numbered 0, 1, 2, ... in op order.  Weights are Q8_0 or F16, 1 <= M <= 8,
 * M*K*(1 or 2 bytes) <= 65536 (above 16384 the program trades weight-ring
 * stages for the wider operand buffer), x rows 16-byte aligned.  Semantics per op
 * are those of vb_matmul_bias. */
typedef struct {
    vb_weight w;
    const float *x;
    int64_t ldx;          /* 0 = K */
    float *y;
    int64_t ldy;          /* 0 = N */
    const float *bias;    /* device F32 [N] or NULL */
    unsigned flags;       /* VB_OUT_BF16 */
    int M;
    int group;
    int wait_group;       /* -1: no dependency */
} vb_gemv_op;

typedef struct vb_program_s *vb_program;
int vb_program_create(vb_ctx *ctx, int n_ops, const vb_gemv_op *ops,
                      vb_program *out);
/* Enqueues one run on the context stream (capturable in a vb_graph). */
int vb_program_run(vb_ctx *ctx, vb_program p);
/* Waits for the stream and reports a device-side error code (a bounded
 * wait that timed out); 0 = OK.  A reported code is cleared, so the program
 * can run again. */
int vb_program_status(vb_ctx *ctx, vb_program p, int *device_error);
void vb_program_destroy(vb_program p);
/* Diagnosis hook for the streaming kernel (programs and the decode step):
 * the number of GPU clock cycles one wait on other CTAs (a grid dependency
 * or a value another CTA writes) may take before the kernel records
 * STREAM_TIMEOUT_GRID (device error 3), stops and exits; 0 restores the
 * default (4e9 cycles, about 2 s).  Waits for the CTA's own weight copies
 * keep the default.  The failure path this exercises (bounded wait, error
 * code, clean exit, a context that stays usable) has no counterpart in the
 * reference, whose host waits on ggml's synchronous compute. */
int vb_set_wait_limit(vb_ctx *ctx, long long cycles);

/* Q8_0 quantization of M rows of K floats into GGUF blocks (34 bytes per
 * 32 values) -- the activation conversion inside every Q8_0 ggml_mul_mat. */
int vb_quantize_q8_0(vb_ctx *ctx, const float *x, int64_t K, int64_t M,
                     void *blocks, int rule);
/* Q8_0 block dequantization (src/model_loader.c:317-331,
 * src/gen_prompt.c:106-125), n values. */
int vb_dequantize_q8_0(vb_ctx *ctx, const void *blocks, int64_t n, float *y);

/* Embedding lookup (gen_forward_text, src/gen_prompt.c:67-131): y row i =
 * row ids[i] of a registered Q8_0 / F16 / F32 table [N rows][K] as F32
 * (Q8_0: (float)qs * d exactly); an id outside [0, N) reads row 0, as the
 * reference does.  ids: device int32 [n]; y: device F32 [n][K], 16-byte
 * aligned; K a multiple of 8.  Replaces the host loop over the F32 copy of
 * embed_tokens made at src/gen_init.c:370-421. */
int vb_get_rows(vb_ctx *ctx, vb_weight table, const int32_t *ids, int64_t n,
                float *y);

/* vcpm_rms_norm (src/minicpm4.c:132-152): with w != NULL and VB_OUT_BF16,
 * y = bf16(bf16(rms_norm(x)) * w); with w == NULL and flags == 0 the plain
 * ggml_rms_norm.  rows of n floats. */
int vb_rms_norm(vb_ctx *ctx, const float *x, const float *w, float *y,
                int64_t n, int64_t rows, float eps, unsigned flags);
/* In-place F32->BF16->F32 (minicpm_bf16_round). */
int vb_bf16_round(vb_ctx *ctx, float *x, int64_t n);
/* y = bf16(a + scale*b) (block residual, src/minicpm4.c:496-528); scale 1
 * skips the multiply as the reference does. */
int vb_residual_add(vb_ctx *ctx, const float *a, const float *b, float scale,
                    float *y, int64_t n, unsigned flags);
/* SwiGLU middle of vcpm_mlp (src/minicpm4.c:441-456):
 * y = bf16(bf16(silu(bf16(g))) * bf16(u)) with VB_OUT_BF16, else silu(g)*u. */
int vb_swiglu(vb_ctx *ctx, const float *g, const float *u, float *y,
              int64_t n, unsigned flags);
/* NEOX rope_ext with the LongRoPE short factors when head_dim == 128
 * (vcpm_rope, src/minicpm4.c:165-223), in place on x[T][n_heads][head_dim];
 * pos: device int32 [T]; VB_OUT_BF16 rounds the result. */
int vb_rope_neox(vb_ctx *ctx, float *x, int head_dim, int n_heads, int T,
                 const int32_t *pos, float theta, unsigned flags);
/* vcpm_fsq_quantize (src/fsq.c:16-29): round(tanh(x)*s)/s, in place. */
int vb_fsq_quantize(vb_ctx *ctx, float *x, int64_t n, float quant_scale);

/* Grouped-query attention over a BF16 K/V store (gqa_group_attn and the
 * per-token loop of vcpm_attention, src/minicpm4.c:232-248,338-412).
 * q: fp32 [T][n_heads][head_dim]; k, v: bf16 [n_kv_heads][n_rows][head_dim];
 * token t attends to rows row_start[t] .. row_start[t]+kv_len[t]-1
 * (row_start, kv_len: device int32 [T]); out: fp32 [T][n_heads*head_dim].
 * Scores are scaled by 1/sqrt(head_dim) and soft-maxed in fp32. */
int vb_attention(vb_ctx *ctx, const float *q, const uint16_t *k,
                 const uint16_t *v, int n_rows, int T, int n_heads,
                 int n_kv_heads, int head_dim, const int32_t *row_start,
                 const int32_t *kv_len, float *out);

/* vb_attention for callers that must not allocate device memory (no
 * counterpart in the reference; this library adds it).  Some hosts cannot
 * let a library call cudaMalloc: an embedding runtime whose own allocator
 * has reserved the GPU's memory up front, or a real-time audio thread that
 * cannot afford the device-wide synchronisation an allocation may cause.
 * vb_attention keeps its per-chunk partial results (when n_rows > 64) in a
 * buffer it grows with cudaMalloc; this variant keeps them instead in a
 * fixed array compiled into the library, VB_ATTENTION_NOALLOC_SCRATCH_BYTES
 * on every GPU that loads the library, held until the process exits.
 * Arguments and results are those of vb_attention; the caller still passes
 * every input and output buffer.  Limit: T * n_heads * ceil(n_rows / 64) *
 * (head_dim + 2) * 4 bytes must not exceed the array size (for example one
 * decode token with 16 heads of 128 over up to 8192 rows fits); larger calls
 * return VB_ERR_INVALID_ARG with the sizes in vb_last_error().  vb_create
 * looks up the array's device address for its context, so a call itself
 * does no set-up.  All calls on a device share the
 * one array: calls that overlap on the GPU (two streams, two contexts of
 * the same device) race and corrupt each other's results.  Nothing in the
 * array needs to start at zero; each call writes every entry it reads. */
#define VB_ATTENTION_NOALLOC_SCRATCH_BYTES (4u << 20)
int vb_attention_noalloc(vb_ctx *ctx, const float *q, const uint16_t *k,
                         const uint16_t *v, int n_rows, int T, int n_heads,
                         int n_kv_heads, int head_dim,
                         const int32_t *row_start, const int32_t *kv_len,
                         float *out);
/* KV-cache append (src/minicpm4.c:299-320): writes bf16(k), bf16(v) of T
 * tokens (fp32 [T][n_kv_heads][head_dim]) into rows dst_row[t] of the
 * bf16 stores [n_kv_heads][n_rows][head_dim]. */
int vb_kv_write(vb_ctx *ctx, const float *k, const float *v, uint16_t *kc,
                uint16_t *vc, int n_rows, int T, int n_kv_heads, int head_dim,
                const int32_t *dst_row);

/* ------------------------------------------------------------------ */
/* Transformer stacks (MiniCPM4 TSLM / RALM / LocDiT blocks / LocEnc) */
/* vcpm_minicpm4_block / vcpm_minicpm4_forward (src/minicpm4.c:467-572)*/
/* ------------------------------------------------------------------ */
typedef struct {
    int hidden, n_heads, n_kv_heads, head_dim, ffn, n_layers;
    float eps;
    float rope_theta;
    int no_rope;         /* RALM: 1 (src/gen_prompt.c:162) */
    float scale_depth;   /* residual scale = scale_depth/sqrt(n_layers) if > 0 */
    int wtype;           /* VB_TYPE_Q8_0 / VB_TYPE_F16 / VB_TYPE_F32 */
} vb_lm_config;

/* Host pointers in GGUF storage; norms are F32 [hidden]. */
typedef struct {
    const void *q, *k, *v, *o, *gate, *up, *down;
    const float *attn_norm, *ffn_norm;
} vb_layer_host;

typedef struct vb_lm vb_lm;
typedef struct vb_kv vb_kv;

int vb_lm_create(vb_ctx *ctx, const vb_lm_config *cfg,
                 const vb_layer_host *layers, const float *final_norm,
                 vb_lm **out);
void vb_lm_destroy(vb_ctx *ctx, vb_lm *lm);
size_t vb_lm_weight_bytes(const vb_lm *lm);

/* BF16 KV cache for n_seqs independent sequences of `capacity` positions
 * (vcpm_kv_cache_init, src/minicpm4.c:93-122; bf16 is exact because the
 * reference rounds K/V to bf16 before caching, src/minicpm4.c:221-222). */
int vb_kv_create(vb_ctx *ctx, const vb_lm *lm, int n_seqs, int capacity,
                 vb_kv **out);
void vb_kv_destroy(vb_ctx *ctx, vb_kv *kv);
int vb_kv_reset(vb_kv *kv, int seq);
int vb_kv_used(const vb_kv *kv, int seq);

/* Causal forward of T tokens for each of n sequences (rows of x are
 * [n][T][hidden], device fp32).  seq: host int32 [n] cache slots; pos: host
 * int32 [n] RoPE position of each sequence's first token (the reference's
 * `pos`, src/minicpm4.c:536-572).  K/V are appended at each sequence's
 * n_used.  out: [n][T][hidden] after the final norm.
 * `final_norm` NULL keeps the final-norm output; hidden states are bf16. */
int vb_lm_forward(vb_ctx *ctx, vb_lm *lm, vb_kv *kv, int n, const int32_t *seq,
                  const int32_t *pos, int T, const float *x, float *out);
/* Bidirectional forward (no_causal = 1, no cache; LocDiT/LocEnc blocks,
 * src/locdit.c:321-370, src/locenc.c:89-113) of n independent segments of
 * T tokens, RoPE positions 0..T-1 in each; no final norm. h in place. */
int vb_lm_forward_noncausal(vb_ctx *ctx, vb_lm *lm, int n, int T, float *h);

/* Single-token decode of a whole stack as ONE persistent-kernel launch: the
 * T = 1 call of vcpm_minicpm4_forward (src/minicpm4.c:536-572) that the
 * reference makes per generated token for the TSLM and the RALM
 * (src/gen_step.c:763, :894).  The decoder binds n KV slots `seq` of `kv`
 * (1 <= n <= 8; n * K bytes of every projection's quantized activation must
 * fit 64 KiB) and owns its buffers, RoPE table (positions below the next
 * power of two >= capacity + 1, at least 512) and launch program.  Q8_0 and
 * F16 stacks.  Each step appends one token per slot exactly as
 * vb_lm_forward(n, seq, pos, T = 1) does; results agree with it within the
 * fp32 accumulation-order tolerance.  x, out: device [n][hidden].  A step is
 * asynchronous; vb_decoder_status synchronises and reports a device-side
 * timeout (the kernel's waits are bounded).  After a reported error the
 * decoder can step again; the failed step's token was still counted in the
 * KV slots (vb_kv_used), which the caller resets or rewinds by prefilling
 * again. */
typedef struct vb_decoder_s *vb_decoder;
int vb_decoder_create(vb_ctx *ctx, vb_lm *lm, vb_kv *kv, int n,
                      const int32_t *seq, vb_decoder *out);
int vb_decoder_step(vb_ctx *ctx, vb_decoder d, const int32_t *pos,
                    const float *x, float *out);
int vb_decoder_status(vb_ctx *ctx, vb_decoder d, int *device_error);
void vb_decoder_destroy(vb_decoder d);

/* ------------------------------------------------------------------ */
/* LocDiT estimator and the CFM loop                                   */
/* (src/locdit.c:140-400, src/gen_step.c:472-652, src/cfm_solver.c)   */
/* ------------------------------------------------------------------ */
typedef struct {
    int hidden, n_layers, n_heads, n_kv_heads, ffn, head_dim;
    int feat_dim, patch;
    float eps;
    int wtype;
} vb_dit_config;

typedef struct {
    const void *in_proj, *cond_proj, *out_proj;
    const float *in_bias, *cond_bias, *out_bias;
    const void *t_w1, *t_w2, *dt_w1, *dt_w2;
    const float *t_b1, *t_b2, *dt_b1, *dt_b2;
    const float *norm;
    const vb_layer_host *layers;
} vb_dit_host;

typedef struct vb_dit vb_dit;

int vb_dit_create(vb_ctx *ctx, const vb_dit_config *cfg, const vb_dit_host *w,
                  vb_dit **out);
void vb_dit_destroy(vb_ctx *ctx, vb_dit *dit);
size_t vb_dit_weight_bytes(const vb_dit *dit);

/* vcpm_locdit_forward for n items: x, cond [n][patch][feat] (device);
 * t, dt: host float [n]; mu: device [n][2*hidden] or NULL; has_mu: host
 * int [n] (0 = unconditional branch, zero mu tokens) or NULL (all 1 when mu
 * is given).  out: device [n][patch][feat]. */
int vb_dit_forward(vb_ctx *ctx, vb_dit *dit, int n, const float *x,
                   const float *cond, const float *t, const float *dt,
                   const float *mu, const int *has_mu, float *out);

/* The Euler CFM solve of vcpm_gen_step (src/gen_step.c:472-652) for n
 * utterances at once: sway t-schedule with the CFG-Zero* skipped steps,
 * cond+uncond evaluated as one batch, CFG-Zero* blend and bf16 Euler update
 * on the device.  mu: device [n][2*hidden] (NULL = no guidance);
 * cond, x: device [n][patch][feat]; x holds the noise on entry and the
 * patch on return. */
int vb_cfm_solve(vb_ctx *ctx, vb_dit *dit, int n, const float *mu,
                 const float *cond, float *x, int n_steps, float cfg_value);

/* ------------------------------------------------------------------ */
/* Autoregressive generation on the device for a batch of utterances  */
/* (src/gen_run.c:60-241, src/gen_prompt.c:186-272,                    */
/*  src/gen_step.c:294-927, src/gen_stop.c:85-230)                      */
/* ------------------------------------------------------------------ */
/* The parts are created beforehand and stay owned by the caller: TSLM and
 * RALM stacks with their final norms, the LocEnc blocks (no final norm;
 * enc_norm is applied to the CLS row), the LocDiT estimator and the
 * projections (weights [K -> N], biases device fp32 or NULL):
 *   enc_in      feat -> enc hidden        enc_to_lm   enc hidden -> hidden
 *   lm_to_dit   hidden -> dit hidden      res_to_dit  hidden -> dit hidden
 *   fsq_in      hidden -> fsq dim         fsq_out     fsq dim -> hidden
 *   fusion      2*hidden -> hidden
 *   stop_proj / stop_head (optional, together): hidden*hidden and hidden*2
 *               values in any registered type, read as the reference's stop
 *               predictor reads them (src/gen_stop.c:126-135,180-195): flat
 *               element j*hidden + i of stop_proj maps input j to output i,
 *               element 2*j + o of stop_head maps input j to class o.  They
 *               are re-laid out once, at vb_gen_create, as exact F32.
 *               stop_head_bias is ignored, as the reference ignores it.
 * enc_special: device [enc hidden] CLS token; enc_norm: device [enc hidden]. */
typedef struct {
    vb_lm *tslm, *ralm, *enc;
    vb_dit *dit;
    vb_weight enc_in, enc_to_lm, lm_to_dit, res_to_dit, fsq_in, fsq_out, fusion, stop_proj, stop_head;
    const float *enc_in_bias, *enc_special, *enc_norm, *enc_to_lm_bias, *lm_to_dit_bias, *res_to_dit_bias,
        *fsq_in_bias, *fsq_out_bias, *fusion_bias, *stop_proj_bias, *stop_head_bias;
    int feat_dim, patch;
    float fsq_scale, eps;
    int cfm_steps;
    float cfg_value;
} vb_gen_parts;

typedef struct vb_gen_s *vb_gen;
/* `batch` utterances (indices 0..batch-1), each with its own KV slots of
 * `max_len` positions; every utterance starts active. */
int vb_gen_create(vb_ctx *ctx, const vb_gen_parts *parts, int batch, int max_len, vb_gen *out);
/* Prompt of T positions per utterance; embeds: device [batch][T][hidden].
 * Resets last_lm_hidden to zero (vcpm_gen_reset, src/gen_init.c:197-198).
 * All utterances must be active.  Grows a prompt buffer owned by the
 * generator when T exceeds every earlier prompt. */
int vb_gen_prefill(vb_ctx *ctx, vb_gen g, int T, const float *embeds);
/* The min_len of vcpm_generation_params (default 2, src/gen_run.c:72): a
 * stop class counts only once n_patches > min_len + 1 (:195-197). */
int vb_gen_set_min_len(vb_gen g, int min_len);
/* One AR step for every ACTIVE utterance (rows in vb_gen_active order):
 * mu -> CFM patch (noise stream seed + utterance index, this step) ->
 * LocEnc -> TSLM -> FSQ -> RALM, then the stop predictor on the hidden saved
 * before the step (gen_predict_stop with the pre-update last_lm_hidden,
 * src/gen_run.c:172-213; the updated hidden when hidden > 2048, as there).
 * patches: device [n_active][patch][feat] or NULL; stop_logits: device
 * [n_active][2] or NULL; stop: device int32 [n_active] or NULL, 1 where the
 * stop class is 1 and the min-length gate is open (the utterance's last
 * patch), else 0.  Stop outputs need stop_proj/stop_head. */
int vb_gen_step_stop(vb_ctx *ctx, vb_gen g, uint64_t seed, float *patches, float *stop_logits, int32_t *stop);
/* vb_gen_step_stop without the stop flags. */
int vb_gen_step(vb_ctx *ctx, vb_gen g, uint64_t seed, float *patches, float *stop_logits);
/* Number of active utterances; their indices in row order into
 * `utterances` (host int32 [batch]) when not NULL.  -1 for a NULL g. */
int vb_gen_active(const vb_gen g, int32_t *utterances);
/* Ends the listed utterances (host int32 indices; retired or unknown-but-in-
 * range indices are ignored): the per-utterance break of src/gen_run.c:208-213
 * for a lockstep batch.  The remaining state rows are compacted so later
 * steps run at the smaller batch; KV slots stay reserved.  Synchronises
 * the context stream. */
int vb_gen_retire(vb_ctx *ctx, vb_gen g, int n, const int32_t *utterances);
/* Copies one state field of the active utterances (row order) into dst,
 * device fp32 [n_active][width] (the fields of vcpm_generate_state,
 * src/generate.h:155-212): */
enum {
    VB_GEN_LM_HIDDEN = 0,        /* lm_hidden_state [hidden]: prompt base[last], then the FSQ output */
    VB_GEN_LAST_LM_HIDDEN = 1,   /* last_lm_hidden [hidden]: the stop predictor's input */
    VB_GEN_RESIDUAL_HIDDEN = 2,  /* residual_hidden_state [hidden] */
    VB_GEN_PREV_PATCH = 3        /* prev_patch [patch*feat] */
};
int vb_gen_state(vb_ctx *ctx, const vb_gen g, int which, float *dst);
void vb_gen_destroy(vb_ctx *ctx, vb_gen g);

/* ---- AudioVAE V2 decoder -------------------------------------------------
 * Latent patches -> 48 kHz PCM, streaming, for a batch of independent
 * utterances decoded in lockstep.  Replaces vcpm_vae_stream_create / _reset
 * / _decode / _free (src/audio_vae_stream.h, src/audio_vae_stream.c:80-619)
 * and the whole-utterance vcpm_vae_v2_decode (src/audio_vae_v2_decoder.c:
 * 149-282, which equals a stream decoded from reset state). */
typedef struct vb_vae_config {
    int latent_dim;     /* latent channels (64) */
    int decoder_dim;    /* 2048: block b maps decoder_dim>>b to decoder_dim>>(b+1)
                         * channels (src/audio_vae_v2.c:40-43); multiple of 256 */
    int rates[6];       /* upsampling strides, transposed-conv kernel 2*rate (8,6,5,2,2,2) */
    int weight_type;    /* storage of the conv weights: VB_TYPE_F32 or VB_TYPE_F16 */
} vb_vae_config;

/* Tensor slots of vb_vae_create, host pointers in GGUF element order.  Conv
 * weights are in cfg.weight_type; biases, Snake alphas and the sr_cond
 * vectors are F32 per channel.  A NULL alpha skips that Snake and a NULL
 * bias adds none (as a missing tensor does in the reference); the sr_cond
 * pair of a block is the bucket row the caller selected (the reference's
 * vcpm_vae_sr_cond_embedding_extract, src/audio_vae_v2.c:652-708) or
 * NULL for none. */
enum {
    VB_VAE_IN_DW_W = 0,    /* audio_vae.decoder.model.0.weight.weight [latent][7] (depthwise) */
    VB_VAE_IN_DW_B = 1,    /* model.0.bias [latent]                                        */
    VB_VAE_IN_PW_W = 2,    /* model.1.weight.weight [D][latent]                             */
    VB_VAE_IN_PW_B = 3,    /* model.1.bias [D]                                              */
    VB_VAE_BLOCK0 = 4,     /* model.(2+b) starts at slot BLOCK0 + b*BLOCK_SLOTS             */
    VB_VAE_BLOCK_SLOTS = 23,
    VB_VAE_B_SR_SCALE = 0, /* sr_cond_model.(2+b).scale_embed row [Ci]                      */
    VB_VAE_B_SR_BIAS = 1,  /* sr_cond_model.(2+b).bias_embed row [Ci]                       */
    VB_VAE_B_ALPHA = 2,    /* model.(2+b).block.0.alpha [Ci]                                */
    VB_VAE_B_UP_W = 3,     /* model.(2+b).block.1.weight.weight [Ci][Co][2*rate]            */
    VB_VAE_B_UP_B = 4,     /* model.(2+b).block.1.bias [Co]                                 */
    VB_VAE_B_RES0 = 5,     /* residual unit u = block.(2+u) at B_RES0 + u*RES_SLOTS         */
    VB_VAE_RES_SLOTS = 6,
    VB_VAE_R_ALPHA0 = 0,   /* block.(2+u).block.0.alpha [Co]                                */
    VB_VAE_R_DW_W = 1,     /* block.(2+u).block.1.weight.weight [Co][7] (depthwise, dilation 1/3/9) */
    VB_VAE_R_DW_B = 2,     /* block.(2+u).block.1.bias [Co]                                 */
    VB_VAE_R_ALPHA2 = 3,   /* block.(2+u).block.2.alpha [Co]                                */
    VB_VAE_R_PW_W = 4,     /* block.(2+u).block.3.weight.weight [Co][Co]                    */
    VB_VAE_R_PW_B = 5,     /* block.(2+u).block.3.bias [Co]                                 */
    VB_VAE_OUT_ALPHA = 142, /* model.8.alpha [D>>6]                                         */
    VB_VAE_OUT_W = 143,     /* model.9.weight.weight [D>>6][7]                              */
    VB_VAE_OUT_B = 144,     /* model.9.bias [1]                                             */
    VB_VAE_N_SLOTS = 145
};

typedef struct vb_vae_s *vb_vae;
typedef struct vb_vae_stream_s *vb_vae_stream;
/* Uploads the decoder (one-time repack to F32 device layouts). */
int vb_vae_create(vb_ctx *ctx, const vb_vae_config *cfg, const void *const *tensors, vb_vae *out);
void vb_vae_destroy(vb_ctx *ctx, vb_vae v);
size_t vb_vae_device_bytes(vb_vae v);
/* History caches of n_streams utterances, zeroed (vcpm_vae_stream_create;
 * patch_size only sets vb_vae_stream_patch_samples). */
int vb_vae_stream_create(vb_ctx *ctx, vb_vae v, int n_streams, int patch_size, vb_vae_stream *out);
int vb_vae_stream_reset(vb_ctx *ctx, vb_vae_stream s);
/* latent: device [n_streams][n_timesteps][latent_dim] (time-major, as
 * vcpm_vae_stream_decode takes it); audio: device [n_streams][n_timesteps *
 * prod(rates)] in (-1, 1).  Both 16-byte aligned.  Enqueued on the context
 * stream; the caches advance by n_timesteps.  The first call, and any call
 * with more timesteps than the stream has seen, (re)allocates the stream's
 * activation buffers (waiting for the stream first). */
int vb_vae_stream_decode(vb_ctx *ctx, vb_vae_stream s, const float *latent, int n_timesteps, float *audio);
/* Ends the listed streams (utterance indices 0..n_streams-1 of the
 * creation; ended or unknown indices are ignored): the VAE side of the
 * per-utterance break of src/gen_run.c:208-213.  The remaining streams'
 * histories are compacted, in utterance order, so later decodes take
 * latent/audio rows of the remaining streams only -- the row order of
 * vb_gen_active after the same vb_gen_retire.  Synchronises the context
 * stream.  vb_vae_stream_reset brings back every stream. */
int vb_vae_stream_retire(vb_ctx *ctx, vb_vae_stream s, int n, const int32_t *utterances);
/* Number of current streams; their utterance indices in row order into
 * `utterances` (host int32 [n_streams]) when not NULL.  -1 for a NULL s. */
int vb_vae_stream_active(vb_vae_stream s, int32_t *utterances);
void vb_vae_stream_destroy(vb_ctx *ctx, vb_vae_stream s);
int vb_vae_stream_conv_cache_count(vb_vae_stream s);     /* 20 */
int vb_vae_stream_upconv_cache_count(vb_vae_stream s);   /* 6  */
int vb_vae_stream_patch_samples(vb_vae_stream s);        /* patch_size * prod(rates) */
size_t vb_vae_stream_state_bytes(vb_vae_stream s);       /* device bytes of the caches */

/* Host helpers restated from the reference for its callers. */
float vb_cfm_sway_t_bf16(int step, int n_steps);   /* src/cfm_solver.c:27-37 */
int vb_cfm_zero_star_steps(int n_steps);           /* src/gen_step.c:50-54 */
void vb_cfm_noise(uint64_t seed, int ar_step, float *x, int n); /* src/gen_step.c:409-431 */
int vb_round_cache_capacity(int required, int model_max); /* src/gen_init.c:115-127 */

#ifdef __cplusplus
}
#endif

#endif /* VCPM_B200_H */
