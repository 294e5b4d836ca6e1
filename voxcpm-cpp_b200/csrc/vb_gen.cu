// vb_gen.cu -- the autoregressive TTS generation loop on the device, for a
// batch of independent utterances stepped in lockstep.  It replays the
// reference's per-patch call order against the library's own entry points:
//
//   prompt   gen_prompt_eval_range (src/gen_prompt.c:186-272):
//            base = TSLM(text embeddings); ralm = RALM(fusion([base; 0]));
//            lm_h = base[last], res_h = ralm[last]
//   per step vcpm_gen_step (src/gen_step.c:294-708) then gen_lm_update
//            (:712-927):
//            mu     = [lm_to_dit(lm_h); res_to_dit(res_h)]             (:318-394)
//            patch  = CFM(noise(seed, step), mu, cond = previous patch)  (:399-652)
//            audio  = enc_to_lm(LocEnc(patch))                          (:209-265)
//            base   = TSLM(audio) (one position)                        (:763)
//            lm_h   = fsq_out(fsq(fsq_in(base)))                        (:268-290)
//            res_h  = RALM(fusion([lm_h; audio])) (one position)        (:864-906)
//            stop   = stop_head(silu(stop_proj(lm_h)))                  (src/gen_stop.c:385-530)
//
// Mat-muls with a batch of B utterances run at M = B (tensor-core path
// from 16 rows); with B <= 2 the single-token TSLM/RALM steps use the
// single-launch decoder.  Every utterance owns its KV slots, state rows and
// noise stream (seed + utterance index), so utterances never interact.
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

// y = bf16(silu(x)) in place (stop-head hidden activation).
__global__ void gen_silu_kernel(float *x, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = bf16r(silu_f(x[i]));
}

}  // namespace vb

using namespace vb;

struct vb_gen_s {
    vb_gen_parts p;
    int B = 0, max_len = 0, ar_step = 0;
    int H = 0, Hr = 0, He = 0, Hd = 0, F = 0, P = 0, FSQ = 0, HS = 0;
    vb_kv *kv = nullptr, *rkv = nullptr;
    vb_decoder dec = nullptr, rdec = nullptr;
    std::vector<int32_t> seq, pos;
    void *mem = nullptr;
    float *fusion_in = nullptr;   // [B][2H]: lm_h | audio_embed
    float *res_h = nullptr, *base = nullptr, *mu = nullptr, *x = nullptr, *prev = nullptr;
    float *enc_seq = nullptr, *enc_cls = nullptr, *fsq = nullptr, *ralm_in = nullptr, *stop_h = nullptr;
    float *noise_host = nullptr;  // pinned [B][P*F]
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

extern "C" void vb_gen_destroy(vb_ctx *ctx, vb_gen g) {
    if (!g) return;
    if (ctx) cudaStreamSynchronize(ctx->stream);
    vb_decoder_destroy(g->dec);
    vb_decoder_destroy(g->rdec);
    vb_kv_destroy(ctx, g->kv);
    vb_kv_destroy(ctx, g->rkv);
    cudaFree(g->mem);
    cudaFreeHost(g->noise_host);
    delete g;
}

extern "C" int vb_gen_create(vb_ctx *ctx, const vb_gen_parts *parts, int batch, int max_len, vb_gen *out) {
    if (!ctx || !parts || !out || batch <= 0 || max_len <= 1) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    const vb_gen_parts &p = *parts;
    if (!p.tslm || !p.ralm || !p.enc || !p.dit || !p.enc_in || !p.enc_to_lm || !p.lm_to_dit || !p.res_to_dit ||
        !p.fsq_in || !p.fsq_out || !p.fusion || !p.enc_special || !p.enc_norm || p.patch <= 0 || p.feat_dim <= 0)
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_create: missing part");
    vb_gen g = new vb_gen_s();
    g->p = p;
    g->B = batch;
    g->max_len = max_len;
    g->H = (int)p.fusion->N;
    g->Hr = g->H;
    g->He = (int)p.enc_in->N;
    g->Hd = (int)p.lm_to_dit->N;
    g->F = p.feat_dim;
    g->P = p.patch;
    g->FSQ = (int)p.fsq_in->N;
    g->HS = p.stop_proj ? (int)p.stop_proj->N : 0;
    const int B = batch, H = g->H, He = g->He, Hd = g->Hd, F = g->F, P = g->P;
    int rc = VB_OK;
    if (p.fusion->K != 2 * H || p.enc_in->K != F || p.enc_to_lm->K != He || p.enc_to_lm->N != H ||
        p.lm_to_dit->K != H || p.res_to_dit->K != H || p.res_to_dit->N != Hd || p.fsq_in->K != H ||
        p.fsq_out->K != g->FSQ || p.fsq_out->N != H)
        rc = set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_create: projection shapes do not chain");
    if (!rc) rc = vb_kv_create(ctx, p.tslm, B, max_len, &g->kv);
    if (!rc) rc = vb_kv_create(ctx, p.ralm, B, max_len, &g->rkv);
    g->seq.resize(B);
    for (int i = 0; i < B; i++) g->seq[i] = i;
    g->pos.assign(B, 0);
    if (!rc && B <= 2) {
        // single-launch decode steps when the batch fits the decoder's operand
        if (vb_decoder_create(ctx, p.tslm, g->kv, B, g->seq.data(), &g->dec) != VB_OK) g->dec = nullptr;
        if (vb_decoder_create(ctx, p.ralm, g->rkv, B, g->seq.data(), &g->rdec) != VB_OK) g->rdec = nullptr;
        ctx->last_error.clear();
    }
    size_t off = 0;
    auto take = [&](size_t floats) {
        const size_t o = off;
        off += (floats * 4 + 255) & ~(size_t)255;
        return o;
    };
    const size_t o_fusion = take((size_t)B * 2 * H), o_res = take((size_t)B * H), o_base = take((size_t)B * H);
    const size_t o_mu = take((size_t)B * 2 * Hd), o_x = take((size_t)B * P * F), o_prev = take((size_t)B * P * F);
    const size_t o_enc = take((size_t)B * (P + 1) * He), o_cls = take((size_t)B * He), o_fsq = take((size_t)B * g->FSQ);
    const size_t o_ralm = take((size_t)B * H), o_stop = take((size_t)B * (g->HS > 0 ? g->HS : 1));
    if (!rc && cudaMalloc(&g->mem, off) != cudaSuccess) rc = set_error(ctx, VB_ERR_OOM, "vb_gen_create: buffers");
    if (!rc && cudaMallocHost(&g->noise_host, (size_t)B * P * F * 4) != cudaSuccess)
        rc = set_error(ctx, VB_ERR_OOM, "vb_gen_create: pinned noise buffer");
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
    cudaMemsetAsync(g->mem, 0, off, ctx->stream);
    *out = g;
    return VB_OK;
}

extern "C" int vb_gen_prefill(vb_ctx *ctx, vb_gen g, int T, const float *embeds) {
    if (!ctx || !g || T <= 0 || !embeds) return VB_ERR_INVALID_ARG;
    const int B = g->B, H = g->H;
    if (g->pos[0] + T > g->max_len) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_prefill: prompt too long");
    // scratch for [B][T] rows: base, fusion input, ralm input/output
    float *buf = nullptr;
    const size_t rows = (size_t)B * T;
    VB_CHECK(ctx, cudaMallocAsync(&buf, rows * H * 4 * 4, ctx->stream));
    float *base = buf, *fin = buf + rows * H, *rin = buf + rows * H * 3;   // fin: [rows][2H]
    int rc = vb_lm_forward(ctx, g->p.tslm, g->kv, B, g->seq.data(), g->pos.data(), T, embeds, base);
    // fusion([base; 0]) for every prompt position
    if (!rc) rc = check_cuda(ctx, cudaMemsetAsync(fin, 0, rows * 2 * H * 4, ctx->stream), "prefill memset");
    if (!rc)
        rc = check_cuda(ctx, cudaMemcpy2DAsync(fin, 2 * H * 4, base, H * 4, H * 4, rows, cudaMemcpyDeviceToDevice,
                                               ctx->stream),
                        "prefill concat");
    if (!rc) rc = gen_mm(ctx, g->p.fusion, fin, (int64_t)rows, 2 * H, rin, H, g->p.fusion_bias);
    if (!rc) rc = vb_lm_forward(ctx, g->p.ralm, g->rkv, B, g->seq.data(), g->pos.data(), T, rin, rin);
    // state: last position of each utterance
    if (!rc)
        rc = check_cuda(ctx, cudaMemcpy2DAsync(g->fusion_in, 2 * H * 4, base + (size_t)(T - 1) * H, (size_t)T * H * 4,
                                               H * 4, B, cudaMemcpyDeviceToDevice, ctx->stream),
                        "prefill lm state");
    if (!rc)
        rc = check_cuda(ctx, cudaMemcpy2DAsync(g->res_h, H * 4, rin + (size_t)(T - 1) * H, (size_t)T * H * 4, H * 4, B,
                                               cudaMemcpyDeviceToDevice, ctx->stream),
                        "prefill ralm state");
    cudaFreeAsync(buf, ctx->stream);
    if (!rc)
        for (int i = 0; i < B; i++) g->pos[i] += T;
    return rc;
}

extern "C" int vb_gen_step(vb_ctx *ctx, vb_gen g, uint64_t seed, float *patches, float *stop_logits) {
    if (!ctx || !g) return VB_ERR_INVALID_ARG;
    const vb_gen_parts &p = g->p;
    const int B = g->B, H = g->H, He = g->He, Hd = g->Hd, F = g->F, P = g->P, PF = P * F;
    if (g->pos[0] + 1 > g->max_len) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_gen_step: cache full");
    float *lm_h = g->fusion_in, *audio = g->fusion_in + H;   // row stride 2H
    int rc;
    // 1. mu = [lm_to_dit(lm_h); res_to_dit(res_h)]
    if ((rc = gen_mm(ctx, p.lm_to_dit, lm_h, B, 2 * H, g->mu, 2 * Hd, p.lm_to_dit_bias))) return rc;
    if ((rc = gen_mm(ctx, p.res_to_dit, g->res_h, B, H, g->mu + Hd, 2 * Hd, p.res_to_dit_bias))) return rc;
    // 2. noise (host SplitMix64 + Box-Muller, per utterance), CFM solve
    for (int i = 0; i < B; i++) vb_cfm_noise(seed + (uint64_t)i, g->ar_step, g->noise_host + (size_t)i * PF, PF);
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
    // 5. FSQ: lm_h = fsq_out(fsq(fsq_in(base)))
    if ((rc = gen_mm(ctx, p.fsq_in, g->base, B, H, g->fsq, g->FSQ, p.fsq_in_bias))) return rc;
    if ((rc = launch_fsq(ctx, g->fsq, (int64_t)B * g->FSQ, p.fsq_scale))) return rc;
    if ((rc = gen_mm(ctx, p.fsq_out, g->fsq, B, g->FSQ, lm_h, 2 * H, p.fsq_out_bias))) return rc;
    // 6. RALM one position over fusion([lm_h; audio])
    if ((rc = gen_mm(ctx, p.fusion, g->fusion_in, B, 2 * H, g->ralm_in, H, p.fusion_bias))) return rc;
    if (g->rdec) rc = vb_decoder_step(ctx, g->rdec, g->pos.data(), g->ralm_in, g->res_h);
    else rc = vb_lm_forward(ctx, p.ralm, g->rkv, B, g->seq.data(), g->pos.data(), 1, g->ralm_in, g->res_h);
    if (rc) return rc;
    // 7. stop head
    if (stop_logits && p.stop_proj && p.stop_head) {
        if ((rc = gen_mm(ctx, p.stop_proj, lm_h, B, 2 * H, g->stop_h, g->HS, p.stop_proj_bias))) return rc;
        gen_silu_kernel<<<(unsigned)(((int64_t)B * g->HS + 255) / 256), 256, 0, ctx->stream>>>(g->stop_h,
                                                                                             (int64_t)B * g->HS);
        VB_LAUNCH_CHECK(ctx, "gen_silu");
        if ((rc = gen_mm(ctx, p.stop_head, g->stop_h, B, g->HS, stop_logits, p.stop_head->N, p.stop_head_bias)))
            return rc;
    }
    for (int i = 0; i < B; i++) g->pos[i] += 1;
    g->ar_step++;
    return VB_OK;
}
