// vb_gen.cu -- the autoregressive TTS generation loop on the device, for a
// batch of independent utterances stepped in lockstep.  It replays the
// reference's per-patch call order against the library's own entry points:
//
//   prompt   gen_prompt_eval_range (src/gen_prompt.c:186-272):
//            base = TSLM(text embeddings); ralm = RALM(fusion([base; 0]));
//            lm_h = base[last], res_h = ralm[last]; last_lm_hidden = 0
//            (vcpm_gen_reset, src/gen_init.c:197-198)
//   per step vcpm_gen_step (src/gen_step.c:294-708) then gen_lm_update
//            (:712-927):
//            mu     = [lm_to_dit(lm_h); res_to_dit(res_h)]             (:318-394)
//            patch  = CFM(noise(seed, step), mu, cond = previous patch)  (:399-652)
//            audio  = enc_to_lm(LocEnc(patch))                          (:209-265)
//            base   = TSLM(audio) (one position)                        (:763)
//            lm_h   = fsq_out(fsq(fsq_in(base)))                        (:268-290)
//            last_lm_hidden = lm_h                                      (:846-848)
//            res_h  = RALM(fusion([lm_h; audio])) (one position)        (:864-906)
//   stop     gen_predict_stop (src/gen_stop.c:85-230) on the hidden
//            saved BEFORE the step (src/gen_run.c:172-183,199-207):
//            logits = H^T silu(W^T h + b), both weights read in their
//            [in][out] storage order as exact F32, no activation
//            quantization, no bf16 rounding, no stop_head bias; class =
//            argmax with class 0 winning ties (:76-81); the class counts
//            only once n_patches > min_len + 1 (src/gen_run.c:195-197).
//
// Mat-muls with B active utterances run at M = B (tensor-core path from 16
// rows); with B <= 2 the single-token TSLM/RALM steps use the single-launch
// decoder.  Every utterance owns its KV slots, state rows and noise stream
// (seed + utterance index), so utterances never interact.  When the host
// retires finished utterances (the break of src/gen_run.c:208-213 per
// utterance), the remaining state rows are compacted so later steps run at
// the smaller M.
#include <algorithm>
#include <vector>

#include "vb_common.cuh"
#include "vb_kernels.cuh"

namespace vb {

// dst row (s*(P+1)) <- special token, for each of B segments.
__global__ void gen_special_rows_kernel(float *seq, const float *special, int B, int P1, int H) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * H) return;
    const int s = (int)(i / H), h = (int)(i % H);
    seq[(int64_t)s * P1 * H + h] = special[h];
}

// fp32 SiLU in place, x / (1 + expf(-x)) without rounding (src/gen_stop.c:174-178).
__global__ void gen_silu_kernel(float *x, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = silu_f(x[i]);
}

// Stop decision per row: argmax of the two logits, class 0 winning ties
// (gen_stop_class_from_logits, src/gen_stop.c:76-81), counted only when
// the min-length gate is open.
__global__ void gen_stop_class_kernel(const float *logits, int n, int gate_open, int32_t *stop) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) stop[i] = (gate_open && logits[2 * i + 1] > logits[2 * i]) ? 1 : 0;
}

// dst row r <- src row map[r] (width floats per row, strides ld).
__global__ void gen_gather_rows_kernel(const float *src, float *dst, const int32_t *map, int rows, int64_t width,
                                       int64_t ld) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * width) return;
    const int64_t r = i / width, c = i % width;
    dst[r * ld + c] = src[(int64_t)map[r] * ld + c];
}

}  // namespace vb

using namespace vb;

struct vb_gen_s {
    vb_gen_parts p;
    int B = 0, n = 0, max_len = 0, ar_step = 0, min_len = 2;
    int H = 0, Hr = 0, He = 0, Hd = 0, F = 0, P = 0, FSQ = 0;
    vb_kv *kv = nullptr, *rkv = nullptr;
    vb_decoder dec = nullptr, rdec = nullptr;
    std::vector<int32_t> seq, pos, utt;   // per active row: KV slot, next position, utterance index
    vb_weight stop_w = nullptr, stop_hw = nullptr;   // F32 [H][H] and [2][H], reference read order
    void *mem = nullptr;
    float *fusion_in = nullptr;   // [B][2H]: lm_h | audio_embed
    float *res_h = nullptr, *base = nullptr, *mu = nullptr, *x = nullptr, *prev = nullptr;
    float *enc_seq = nullptr, *enc_cls = nullptr, *fsq = nullptr, *ralm_in = nullptr, *stop_h = nullptr;
    float *last_lm = nullptr;     // [B][H]: last_lm_hidden, the stop predictor's input
    float *stop_l = nullptr;      // [B][2]: logits when the caller passes none
    float *tmp = nullptr;         // [B][2H]: row compaction staging
    int32_t *map_dev = nullptr;   // [B]: row map of a compaction
    int32_t *map_host = nullptr;  // pinned [B]
    float *noise_host = nullptr;  // pinned [B][P*F]
    vb::Arena prompt;             // prefill rows, grown only by vb_gen_prefill
};

static int gen_mm(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, float *y, int64_t ldy,
                  const float *bias, unsigned flags = 0, int64_t seg = 0, int64_t seg_stride = 0,
                  int64_t seg_off = 0) {
    MatmulOut o;
    o.y = y;
    o.ldy = ldy;
    o.bias = bias;
    o.flags = flags;
    o.seg = seg;
    o.seg_stride = seg_stride;
    o.seg_off = seg_off;
    return launch_matmul(ctx, w, x, M, ldx, 0, o);
}

static void gen_free_decoders(vb_gen g) {
    vb_decoder_destroy(g->dec);
    vb_decoder_destroy(g->rdec);
    g->dec = g->rdec = nullptr;
}

// Single-launch decode steps for batches of up to four utterances, where
// they beat the per-op stack (B200, 28-layer step: 1.1 / 1.7 / 2.2 / 2.6 ms
// at 1-4 sequences against 2.3-2.7 ms; from six on the per-op stack's
// tensor-core GEMMs win); larger batches take the per-op stack.
static void gen_make_decoders(vb_ctx *ctx, vb_gen g) {
    gen_free_decoders(g);
    if (g->n < 1 || g->n > 4) return;
    const std::string keep = ctx->last_error;
    if (vb_decoder_create(ctx, g->p.tslm, g->kv, g->n, g->seq.data(), &g->dec) != VB_OK) g->dec = nullptr;
    if (vb_decoder_create(ctx, g->p.ralm, g->rkv, g->n, g->seq.data(), &g->rdec) != VB_OK) g->rdec = nullptr;
    ctx->last_error = keep;
}

extern "C" void vb_gen_destroy(vb_ctx *ctx, vb_gen g) {
    if (!g) return;
    if (ctx) cudaStreamSynchronize(ctx->stream);
    gen_free_decoders(g);
    vb_kv_destroy(ctx, g->kv);
    vb_kv_destroy(ctx, g->rkv);
    weight_free(ctx, g->stop_w);
    weight_free(ctx, g->stop_hw);
    cudaFree(g->mem);
    cudaFree(g->prompt.ptr);
    cudaFreeHost(g->noise_host);
    cudaFreeHost(g->map_host);
    delete g;
}

extern "C" int vb_gen_create(vb_ctx *ctx, const vb_gen_parts *parts, int batch, int max_len, vb_gen *out) {
    if (!ctx || !parts || !out || batch <= 0 || max_len <= 1) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    const vb_gen_parts &p = *parts;
    if (!p.tslm || !p.ralm || !p.enc || !p.dit || !p.enc_in || !p.enc_to_lm || !p.lm_to_dit || !p.res_to_dit ||
        !p.fsq_in || !p.fsq_out || !p.fusion || !p.enc_special || !p.enc_norm || p.patch <= 0 || p.feat_dim <= 0)
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_create: missing part");
    if (!p.stop_proj != !p.stop_head)
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_create: stop_proj and stop_head come together");
    vb_gen g = new vb_gen_s();
    g->p = p;
    g->B = g->n = batch;
    g->max_len = max_len;
    g->H = (int)p.fusion->N;
    g->Hr = g->H;
    g->He = (int)p.enc_in->N;
    g->Hd = (int)p.lm_to_dit->N;
    g->F = p.feat_dim;
    g->P = p.patch;
    g->FSQ = (int)p.fsq_in->N;
    const int B = batch, H = g->H, He = g->He, Hd = g->Hd, F = g->F, P = g->P;
    int rc = VB_OK;
    if (p.fusion->K != 2 * H || p.enc_in->K != F || p.enc_to_lm->K != He || p.enc_to_lm->N != H ||
        p.lm_to_dit->K != H || p.res_to_dit->K != H || p.res_to_dit->N != Hd || p.fsq_in->K != H ||
        p.fsq_out->K != g->FSQ || p.fsq_out->N != H)
        rc = set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_create: projection shapes do not chain");
    // stop_proj holds hidden x hidden values, stop_head hidden x 2 (the reference's hs = hidden_size)
    if (!rc && p.stop_proj) rc = weight_transpose_f32(ctx, p.stop_proj, H, H, &g->stop_w);
    if (!rc && p.stop_head) rc = weight_transpose_f32(ctx, p.stop_head, H, 2, &g->stop_hw);
    if (!rc) rc = vb_kv_create(ctx, p.tslm, B, max_len, &g->kv);
    if (!rc) rc = vb_kv_create(ctx, p.ralm, B, max_len, &g->rkv);
    g->seq.resize(B);
    g->utt.resize(B);
    for (int i = 0; i < B; i++) g->seq[i] = g->utt[i] = i;
    g->pos.assign(B, 0);
    if (!rc) gen_make_decoders(ctx, g);
    size_t off = 0;
    auto take = [&](size_t floats) {
        const size_t o = off;
        off += (floats * 4 + 255) & ~(size_t)255;
        return o;
    };
    const size_t o_fusion = take((size_t)B * 2 * H), o_res = take((size_t)B * H), o_base = take((size_t)B * H);
    const size_t o_mu = take((size_t)B * 2 * Hd), o_x = take((size_t)B * P * F), o_prev = take((size_t)B * P * F);
    const size_t o_enc = take((size_t)B * (P + 1) * He), o_cls = take((size_t)B * He), o_fsq = take((size_t)B * g->FSQ);
    const size_t o_ralm = take((size_t)B * H), o_stop = take((size_t)B * H), o_last = take((size_t)B * H);
    const size_t o_sl = take((size_t)B * 2);
    const size_t o_tmp = take((size_t)B * std::max(2 * H, P * F)), o_map = take((size_t)B);
    if (!rc && cudaMalloc(&g->mem, off) != cudaSuccess) rc = set_error(ctx, VB_ERR_OOM, "vb_gen_create: buffers");
    if (!rc && cudaMallocHost(&g->noise_host, (size_t)B * P * F * 4) != cudaSuccess)
        rc = set_error(ctx, VB_ERR_OOM, "vb_gen_create: pinned noise buffer");
    if (!rc && cudaMallocHost(&g->map_host, (size_t)B * 4) != cudaSuccess)
        rc = set_error(ctx, VB_ERR_OOM, "vb_gen_create: pinned row map");
    if (!rc) rc = check_cuda(ctx, cudaMemsetAsync(g->mem, 0, off, ctx->stream), "vb_gen_create: clear");
    if (rc) {
        vb_gen_destroy(ctx, g);
        return rc;
    }
    uint8_t *m = (uint8_t *)g->mem;
    g->fusion_in = (float *)(m + o_fusion);
    g->res_h = (float *)(m + o_res);
    g->base = (float *)(m + o_base);
    g->mu = (float *)(m + o_mu);
    g->x = (float *)(m + o_x);
    g->prev = (float *)(m + o_prev);
    g->enc_seq = (float *)(m + o_enc);
    g->enc_cls = (float *)(m + o_cls);
    g->fsq = (float *)(m + o_fsq);
    g->ralm_in = (float *)(m + o_ralm);
    g->stop_h = (float *)(m + o_stop);
    g->last_lm = (float *)(m + o_last);
    g->stop_l = (float *)(m + o_sl);
    g->tmp = (float *)(m + o_tmp);
    g->map_dev = (int32_t *)(m + o_map);
    *out = g;
    return VB_OK;
}

extern "C" int vb_gen_set_min_len(vb_gen g, int min_len) {
    if (!g) return VB_ERR_INVALID_ARG;
    g->min_len = min_len;
    return VB_OK;
}

extern "C" int vb_gen_prefill(vb_ctx *ctx, vb_gen g, int T, const float *embeds) {
    if (!ctx || !g || T <= 0 || !embeds) return VB_ERR_INVALID_ARG;
    const int B = g->B, H = g->H;
    if (g->n != B) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_prefill: utterances were retired");
    if (g->pos[0] + T > g->max_len) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_prefill: prompt too long");
    // rows [B][T]: base, fusion input [2H], ralm input/output
    const size_t rows = (size_t)B * T;
    int rc = arena_reserve(ctx, g->prompt, rows * H * 4 * 4);
    if (rc) return rc;
    float *buf = (float *)g->prompt.ptr;
    float *base = buf, *fin = buf + rows * H, *rin = buf + rows * H * 3;   // fin: [rows][2H]
    rc = vb_lm_forward(ctx, g->p.tslm, g->kv, B, g->seq.data(), g->pos.data(), T, embeds, base);
    // fusion([base; 0]) for every prompt position
    if (!rc) rc = check_cuda(ctx, cudaMemsetAsync(fin, 0, rows * 2 * H * 4, ctx->stream), "prefill memset");
    if (!rc)
        rc = check_cuda(ctx, cudaMemcpy2DAsync(fin, 2 * H * 4, base, H * 4, H * 4, rows, cudaMemcpyDeviceToDevice,
                                               ctx->stream),
                        "prefill concat");
    if (!rc) rc = gen_mm(ctx, g->p.fusion, fin, (int64_t)rows, 2 * H, rin, H, g->p.fusion_bias);
    if (!rc) rc = vb_lm_forward(ctx, g->p.ralm, g->rkv, B, g->seq.data(), g->pos.data(), T, rin, rin);
    // state: last position of each utterance; last_lm_hidden starts at zero
    if (!rc)
        rc = check_cuda(ctx, cudaMemcpy2DAsync(g->fusion_in, 2 * H * 4, base + (size_t)(T - 1) * H, (size_t)T * H * 4,
                                               H * 4, B, cudaMemcpyDeviceToDevice, ctx->stream),
                        "prefill lm state");
    if (!rc)
        rc = check_cuda(ctx, cudaMemcpy2DAsync(g->res_h, H * 4, rin + (size_t)(T - 1) * H, (size_t)T * H * 4, H * 4, B,
                                               cudaMemcpyDeviceToDevice, ctx->stream),
                        "prefill ralm state");
    if (!rc) rc = check_cuda(ctx, cudaMemsetAsync(g->last_lm, 0, (size_t)B * H * 4, ctx->stream), "prefill reset");
    if (!rc)
        for (int i = 0; i < B; i++) g->pos[i] += T;
    return rc;
}

// gen_predict_stop for the n active rows of `hidden` (row stride ldh):
// logits [n][2], stop flags [n] when asked for.
static int gen_stop(vb_ctx *ctx, vb_gen g, const float *hidden, int64_t ldh, float *logits, int32_t *stop) {
    const int n = g->n, H = g->H;
    int rc = gen_mm(ctx, g->stop_w, hidden, n, ldh, g->stop_h, H, g->p.stop_proj_bias);
    if (rc) return rc;
    gen_silu_kernel<<<(unsigned)(((int64_t)n * H + 255) / 256), 256, 0, ctx->stream>>>(g->stop_h, (int64_t)n * H);
    VB_LAUNCH_CHECK(ctx, "gen_silu");
    if ((rc = gen_mm(ctx, g->stop_hw, g->stop_h, n, H, logits, 2, nullptr))) return rc;
    if (stop) {
        // n_patches after this step is ar_step + 1 (src/gen_run.c:195-197)
        const int gate_open = (g->ar_step + 1) > g->min_len + 1;
        gen_stop_class_kernel<<<(unsigned)((n + 127) / 128), 128, 0, ctx->stream>>>(logits, n, gate_open, stop);
        VB_LAUNCH_CHECK(ctx, "gen_stop_class");
    }
    return VB_OK;
}

extern "C" int vb_gen_step_stop(vb_ctx *ctx, vb_gen g, uint64_t seed, float *patches, float *stop_logits,
                                int32_t *stop) {
    if (!ctx || !g) return VB_ERR_INVALID_ARG;
    const vb_gen_parts &p = g->p;
    const int B = g->n, H = g->H, He = g->He, Hd = g->Hd, F = g->F, P = g->P, PF = P * F;
    if (B == 0) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_step: every utterance is retired");
    if ((stop_logits || stop) && !g->stop_w)
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_step: stop outputs need stop_proj and stop_head");
    for (int i = 0; i < B; i++)
        if (g->pos[i] + 1 > g->max_len) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_step: cache full");
    float *lm_h = g->fusion_in, *audio = g->fusion_in + H;   // row stride 2H
    float *logits = stop_logits ? stop_logits : g->stop_l;
    // the stop predictor reads last_lm_hidden as it was before this step when
    // hidden_size <= 2048 (the saved copy of src/gen_run.c:178-183), else the
    // updated one (the reference then has no copy)
    const bool want_stop = stop_logits || stop;
    const bool stop_pre = H <= 2048;
    int rc;
    if (want_stop && stop_pre && (rc = gen_stop(ctx, g, g->last_lm, H, logits, stop))) return rc;
    // 1. mu = [lm_to_dit(lm_h); res_to_dit(res_h)]
    if ((rc = gen_mm(ctx, p.lm_to_dit, lm_h, B, 2 * H, g->mu, 2 * Hd, p.lm_to_dit_bias))) return rc;
    if ((rc = gen_mm(ctx, p.res_to_dit, g->res_h, B, H, g->mu + Hd, 2 * Hd, p.res_to_dit_bias))) return rc;
    // 2. noise (host SplitMix64 + Box-Muller, per utterance), CFM solve
    for (int i = 0; i < B; i++)
        vb_cfm_noise(seed + (uint64_t)g->utt[i], g->ar_step, g->noise_host + (size_t)i * PF, PF);
    VB_CHECK(ctx, cudaMemcpyAsync(g->x, g->noise_host, (size_t)B * PF * 4, cudaMemcpyHostToDevice, ctx->stream));
    if ((rc = vb_cfm_solve(ctx, p.dit, B, g->mu, g->prev, g->x, p.cfm_steps, p.cfg_value))) return rc;
    VB_CHECK(ctx, cudaMemcpyAsync(g->prev, g->x, (size_t)B * PF * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    if (patches)
        VB_CHECK(ctx, cudaMemcpyAsync(patches, g->x, (size_t)B * PF * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    // 3. LocEnc over [special; in_proj(patch)] -> norm(CLS) -> enc_to_lm
    gen_special_rows_kernel<<<(unsigned)(((int64_t)B * He + 255) / 256), 256, 0, ctx->stream>>>(g->enc_seq,
                                                                                             p.enc_special, B, P + 1,
                                                                                             He);
    VB_LAUNCH_CHECK(ctx, "gen_special_rows");
    if ((rc = gen_mm(ctx, p.enc_in, g->prev, (int64_t)B * P, F, g->enc_seq, He, p.enc_in_bias, 0, P, P + 1, 1)))
        return rc;
    if ((rc = vb_lm_forward_noncausal(ctx, p.enc, B, P + 1, g->enc_seq))) return rc;
    if ((rc = launch_rms_norm(ctx, g->enc_seq, p.enc_norm, g->enc_cls, He, B, p.eps, VB_OUT_BF16, (int64_t)(P + 1) * He,
                              He)))
        return rc;
    if ((rc = gen_mm(ctx, p.enc_to_lm, g->enc_cls, B, He, audio, 2 * H, p.enc_to_lm_bias))) return rc;
    // 4. TSLM one position; the decoder takes a packed [B][H] input
    VB_CHECK(ctx, cudaMemcpy2DAsync(g->ralm_in, H * 4, audio, 2 * H * 4, H * 4, B, cudaMemcpyDeviceToDevice,
                                    ctx->stream));
    if (g->dec) rc = vb_decoder_step(ctx, g->dec, g->pos.data(), g->ralm_in, g->base);
    else rc = vb_lm_forward(ctx, p.tslm, g->kv, B, g->seq.data(), g->pos.data(), 1, g->ralm_in, g->base);
    if (rc) return rc;
    // 5. FSQ: lm_h = fsq_out(fsq(fsq_in(base))); last_lm_hidden = lm_h
    if ((rc = gen_mm(ctx, p.fsq_in, g->base, B, H, g->fsq, g->FSQ, p.fsq_in_bias))) return rc;
    if ((rc = launch_fsq(ctx, g->fsq, (int64_t)B * g->FSQ, p.fsq_scale))) return rc;
    if ((rc = gen_mm(ctx, p.fsq_out, g->fsq, B, g->FSQ, lm_h, 2 * H, p.fsq_out_bias))) return rc;
    VB_CHECK(ctx, cudaMemcpy2DAsync(g->last_lm, H * 4, lm_h, 2 * H * 4, H * 4, B, cudaMemcpyDeviceToDevice,
                                    ctx->stream));
    // 6. RALM one position over fusion([lm_h; audio])
    if ((rc = gen_mm(ctx, p.fusion, g->fusion_in, B, 2 * H, g->ralm_in, H, p.fusion_bias))) return rc;
    if (g->rdec) rc = vb_decoder_step(ctx, g->rdec, g->pos.data(), g->ralm_in, g->res_h);
    else rc = vb_lm_forward(ctx, p.ralm, g->rkv, B, g->seq.data(), g->pos.data(), 1, g->ralm_in, g->res_h);
    if (rc) return rc;
    // 7. stop predictor on the updated hidden (hidden_size > 2048 only)
    if (want_stop && !stop_pre && (rc = gen_stop(ctx, g, g->last_lm, H, logits, stop))) return rc;
    for (int i = 0; i < B; i++) g->pos[i] += 1;
    g->ar_step++;
    return VB_OK;
}

extern "C" int vb_gen_step(vb_ctx *ctx, vb_gen g, uint64_t seed, float *patches, float *stop_logits) {
    return vb_gen_step_stop(ctx, g, seed, patches, stop_logits, nullptr);
}

extern "C" int vb_gen_active(const vb_gen g, int32_t *utterances) {
    if (!g) return -1;
    if (utterances)
        for (int i = 0; i < g->n; i++) utterances[i] = g->utt[i];
    return g->n;
}

extern "C" int vb_gen_retire(vb_ctx *ctx, vb_gen g, int n, const int32_t *utterances) {
    if (!ctx || !g || n < 0 || (n > 0 && !utterances)) return VB_ERR_INVALID_ARG;
    std::vector<char> drop(g->B, 0);
    for (int i = 0; i < n; i++) {
        const int u = utterances[i];
        if (u < 0 || u >= g->B) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_retire: utterance %d out of range", u);
        drop[u] = 1;
    }
    std::vector<int32_t> keep;
    for (int r = 0; r < g->n; r++)
        if (!drop[g->utt[r]]) keep.push_back(r);
    if ((int)keep.size() == g->n) return VB_OK;
    const int nk = (int)keep.size();
    if (nk > 0) {
        // the pinned row map may still feed an earlier compaction's copy
        VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
        std::copy(keep.begin(), keep.end(), g->map_host);
        VB_CHECK(ctx, cudaMemcpyAsync(g->map_dev, g->map_host, (size_t)nk * 4, cudaMemcpyHostToDevice, ctx->stream));
        const int H = g->H, PF = g->P * g->F;
        struct Rows { float *buf; int64_t width; };
        const Rows state[] = {{g->fusion_in, 2 * (int64_t)H}, {g->res_h, H}, {g->prev, PF}, {g->last_lm, H}};
        for (const Rows &s : state) {
            const int64_t total = (int64_t)nk * s.width;
            gen_gather_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, ctx->stream>>>(s.buf, g->tmp, g->map_dev,
                                                                                            nk, s.width, s.width);
            VB_LAUNCH_CHECK(ctx, "gen_gather_rows");
            VB_CHECK(ctx, cudaMemcpyAsync(s.buf, g->tmp, (size_t)total * 4, cudaMemcpyDeviceToDevice, ctx->stream));
        }
    }
    std::vector<int32_t> seq(nk), pos(nk), utt(nk);
    for (int i = 0; i < nk; i++) {
        seq[i] = g->seq[keep[i]];
        pos[i] = g->pos[keep[i]];
        utt[i] = g->utt[keep[i]];
    }
    g->seq = seq;
    g->pos = pos;
    g->utt = utt;
    g->n = nk;
    VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
    gen_make_decoders(ctx, g);
    return VB_OK;
}

extern "C" int vb_gen_state(vb_ctx *ctx, const vb_gen g, int which, float *dst) {
    if (!ctx || !g || !dst) return VB_ERR_INVALID_ARG;
    const int H = g->H, n = g->n;
    const float *src;
    int64_t width, ld;
    switch (which) {
        case VB_GEN_LM_HIDDEN: src = g->fusion_in; width = H; ld = 2 * (int64_t)H; break;
        case VB_GEN_LAST_LM_HIDDEN: src = g->last_lm; width = H; ld = H; break;
        case VB_GEN_RESIDUAL_HIDDEN: src = g->res_h; width = H; ld = H; break;
        case VB_GEN_PREV_PATCH: src = g->prev; width = (int64_t)g->P * g->F; ld = width; break;
        default: return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_state: unknown field %d", which);
    }
    if (n == 0) return VB_OK;
    VB_CHECK(ctx, cudaMemcpy2DAsync(dst, (size_t)width * 4, src, (size_t)ld * 4, (size_t)width * 4, n,
                                    cudaMemcpyDeviceToDevice, ctx->stream));
    return VB_OK;
}
