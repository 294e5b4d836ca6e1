// vb_attn.cu -- grouped-query attention over a BF16 K/V store.
//
// Semantics of gqa_group_attn / vcpm_attention (src/minicpm4.c:232-412):
// for token t and query head h of KV group g = h / (n_heads/n_kv),
//   s_l = (q . k_l) * (1/sqrt(head_dim)),  p = softmax(s),  o = sum_l p_l v_l
// over the rows row_start[t] .. row_start[t]+kv_len[t]-1 of the group's
// K/V (causal decode/prefill: the sequence's cache prefix; bidirectional
// LocDiT/LocEnc: the segment's fresh K/V).  K/V hold bf16 values (the
// reference rounds them to bf16 before caching), q is fp32.
//
// Mapping: grid (chunks, n_kv, T); a CTA stages one chunk of ATT_CH K/V rows
// of one group in shared memory (rows padded to an odd word count so the
// per-lane row reads are bank-conflict free) and each warp handles one query
// head of the group: lanes own positions for the scores, then dimensions for
// the value sum.  With one chunk the CTA writes the normalised output; with
// several it writes (max, sum, partial output) to scratch and a combine pass
// merges the chunks (flash-decoding).
#include "vb_common.cuh"
#include "vb_kernels.cuh"


namespace vb {

constexpr int ATT_CH = 64;         // K/V rows per CTA
constexpr int ATT_WARPS = 8;
constexpr int ATT_HD_MAX = 256;
constexpr int ATT_LD = 4;           // 16-byte K and V loads per thread in flight while staging a chunk

struct AttnArgs {
    const float *q;
    int64_t ldq;
    const uint16_t *k, *v;
    int n_rows, n_heads, n_kv, head_dim, n_chunks;
    const int32_t *row_start, *kv_len;
    float *out;
    int64_t ldo;
    float *part;     // [T][n_heads][n_chunks][head_dim + 2] when n_chunks > 1
    float kq_scale;
};

__global__ void __launch_bounds__(ATT_WARPS * 32) attn_chunk_kernel(AttnArgs a) {
    extern __shared__ __align__(16) uint32_t sm[];
    const int c = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
    const int HD = a.head_dim, HW = HD >> 1;
    const int rw = (HW & 1) ? HW : HW + 1;             // padded row words
    const int qpk = a.n_heads / a.n_kv;
    uint32_t *ks = sm;                                  // [ATT_CH][rw]
    uint32_t *vs = ks + ATT_CH * rw;                    // [ATT_CH][rw]
    float *qs = reinterpret_cast<float *>(vs + ATT_CH * rw);   // [qpk][HD]
    float *es = qs + qpk * HD;                          // [ATT_WARPS][ATT_CH]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int L = a.kv_len[t];
    const int p0 = c * ATT_CH;
    const int n = min(ATT_CH, L - p0);
    if (n <= 0) {   // this token has fewer rows than the widest token
        if (!a.part) return;
        for (int j = warp; j < qpk; j += ATT_WARPS) {
            float *pp = a.part + (((int64_t)t * a.n_heads + g * qpk + j) * a.n_chunks + c) * (HD + 2);
            for (int d = lane; d < HD + 2; d += 32) pp[d] = (d == 0) ? -INFINITY : 0.0f;
        }
        return;
    }
    const int64_t base = ((int64_t)g * a.n_rows + a.row_start[t] + p0) * HW;
    const uint32_t *kg = reinterpret_cast<const uint32_t *>(a.k) + base;
    const uint32_t *vg = reinterpret_cast<const uint32_t *>(a.v) + base;
    if ((HW & 3) == 0) {
        // 16-byte loads, a batch of ATT_LD per thread in flight before any
        // store (rows are 16-byte aligned in global memory, padded in shared)
        const uint4 *kg4 = reinterpret_cast<const uint4 *>(kg), *vg4 = reinterpret_cast<const uint4 *>(vg);
        const int w4 = (n * HW) >> 2;
        for (int i0 = threadIdx.x; i0 < w4; i0 += ATT_LD * blockDim.x) {
            uint4 kk[ATT_LD], vv[ATT_LD];
#pragma unroll
            for (int u = 0; u < ATT_LD; u++) {
                const int i = i0 + u * blockDim.x;
                if (i < w4) {
                    kk[u] = __ldg(kg4 + i);
                    vv[u] = __ldg(vg4 + i);
                }
            }
#pragma unroll
            for (int u = 0; u < ATT_LD; u++) {
                const int i = i0 + u * blockDim.x;
                if (i < w4) {
                    const int r = (4 * i) / HW, w = (4 * i) % HW;
                    uint32_t *kd = ks + r * rw + w, *vd = vs + r * rw + w;
                    kd[0] = kk[u].x; kd[1] = kk[u].y; kd[2] = kk[u].z; kd[3] = kk[u].w;
                    vd[0] = vv[u].x; vd[1] = vv[u].y; vd[2] = vv[u].z; vd[3] = vv[u].w;
                }
            }
        }
    } else {
        for (int i = threadIdx.x; i < n * HW; i += blockDim.x) {
            const int r = i / HW, w = i % HW;
            ks[r * rw + w] = __ldg(kg + i);
            vs[r * rw + w] = __ldg(vg + i);
        }
    }
    for (int i = threadIdx.x; i < qpk * HD; i += blockDim.x) {
        const int j = i / HD, d = i % HD;
        qs[i] = a.q[(int64_t)t * a.ldq + (int64_t)(g * qpk + j) * HD + d];
    }
    __syncthreads();

    for (int j = warp; j < qpk; j += ATT_WARPS) {
        const float *qv = qs + j * HD;
        float *e = es + warp * ATT_CH;
        // scores: lane owns positions lane, lane+32
        float s[ATT_CH / 32];
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < ATT_CH / 32; u++) {
            const int p = lane + 32 * u;
            float acc = -INFINITY;
            if (p < n) {
                acc = 0.0f;
                const uint32_t *kr = ks + p * rw;
                for (int w = 0; w < HW; w++) {
                    const uint32_t kk = kr[w];
                    acc = fmaf(__uint_as_float(kk << 16), qv[2 * w], acc);
                    acc = fmaf(__uint_as_float(kk & 0xffff0000u), qv[2 * w + 1], acc);
                }
                acc = __fmul_rn(acc, a.kq_scale);
            }
            s[u] = acc;
            mx = fmaxf(mx, acc);
        }
        mx = warp_max(mx);
        float l = 0.0f;
#pragma unroll
        for (int u = 0; u < ATT_CH / 32; u++) {
            const int p = lane + 32 * u;
            const float ev = (p < n) ? expf(s[u] - mx) : 0.0f;
            e[p] = ev;
            l += ev;
        }
        l = warp_sum(l);
        __syncwarp();
        // values: lane owns dimensions lane, lane+32, ...
        float o[ATT_HD_MAX / 32];
#pragma unroll
        for (int u = 0; u < ATT_HD_MAX / 32; u++) o[u] = 0.0f;
        for (int p = 0; p < n; p++) {
            const float ep = e[p];
            const uint32_t *vr = vs + p * rw;
#pragma unroll
            for (int u = 0; u < ATT_HD_MAX / 32; u++) {
                const int d = lane + 32 * u;
                if (d < HD) {
                    const uint32_t vv = vr[d >> 1];
                    const float vf = __uint_as_float((d & 1) ? (vv & 0xffff0000u) : (vv << 16));
                    o[u] = fmaf(ep, vf, o[u]);
                }
            }
        }
        const int h = g * qpk + j;
        if (a.n_chunks == 1) {
            float *dst = a.out + (int64_t)t * a.ldo + (int64_t)h * HD;
#pragma unroll
            for (int u = 0; u < ATT_HD_MAX / 32; u++) {
                const int d = lane + 32 * u;
                if (d < HD) dst[d] = __fdiv_rn(o[u], l);
            }
        } else {
            float *pp = a.part + (((int64_t)t * a.n_heads + h) * a.n_chunks + c) * (HD + 2);
            if (lane == 0) { pp[0] = mx; pp[1] = l; }
#pragma unroll
            for (int u = 0; u < ATT_HD_MAX / 32; u++) {
                const int d = lane + 32 * u;
                if (d < HD) pp[2 + d] = o[u];
            }
        }
        __syncwarp();
    }
}

// Bidirectional segments of T <= 32 tokens (LocDiT, LocEnc): one CTA per
// (KV group, segment) stages the segment's K/V rows once (bf16 -> fp32 in
// shared memory) and its warps take the group's (token, query head) pairs.
// A lane owns head dimensions lane, lane + 32, ...: each score is the warp
// sum of the lanes' partial dot products, so all 32 lanes work on every key
// (T is well below 32 here).  Scores scaled by 1/sqrt(head_dim), softmax
// with expf in fp32, the output divided by the sum (IEEE division).
template <int DPL>   // head_dim / 32
__global__ void __launch_bounds__(ATT_WARPS * 32) attn_segment_kernel(AttnArgs a, int T) {
    extern __shared__ __align__(16) float smf[];
    constexpr int HD = DPL * 32;
    const int g = blockIdx.x, sgi = blockIdx.y;
    const int qpk = a.n_heads / a.n_kv;
    float *ks = smf;              // [T][HD]
    float *vs = ks + T * HD;      // [T][HD]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = ((int64_t)g * a.n_rows + (int64_t)sgi * T) * HD;
    for (int i = threadIdx.x; i < T * HD; i += blockDim.x) {
        ks[i] = bf16_to_f(a.k[base + i]);
        vs[i] = bf16_to_f(a.v[base + i]);
    }
    __syncthreads();
    // blockIdx.z picks this CTA's ATT_WARPS (token, head) rows of the segment
    for (int pr = blockIdx.z * ATT_WARPS + warp; pr < T * qpk; pr += ATT_WARPS * gridDim.z) {
        const int t = pr / qpk, h = g * qpk + pr % qpk;
        const int64_t tok = (int64_t)sgi * T + t;
        const float *qr = a.q + tok * a.ldq + (int64_t)h * HD;
        float qv[DPL];
#pragma unroll
        for (int u = 0; u < DPL; u++) qv[u] = qr[lane + 32 * u];
        float sc[32];
        float mx = -INFINITY;
#pragma unroll
        for (int p = 0; p < 32; p++) {
            if (p < T) {                       // uniform over the warp
                float part = 0.0f;
#pragma unroll
                for (int u = 0; u < DPL; u++) part = fmaf(qv[u], ks[p * HD + lane + 32 * u], part);
                const float sp = __fmul_rn(warp_sum(part), a.kq_scale);
                sc[p] = sp;
                mx = fmaxf(mx, sp);
            }
        }
        float l = 0.0f, o[DPL];
#pragma unroll
        for (int u = 0; u < DPL; u++) o[u] = 0.0f;
#pragma unroll
        for (int p = 0; p < 32; p++) {
            if (p < T) {
                const float ep = expf(sc[p] - mx);
                l += ep;
#pragma unroll
                for (int u = 0; u < DPL; u++) o[u] = fmaf(ep, vs[p * HD + lane + 32 * u], o[u]);
            }
        }
        float *dst = a.out + tok * a.ldo + (int64_t)h * HD;
#pragma unroll
        for (int u = 0; u < DPL; u++) dst[lane + 32 * u] = __fdiv_rn(o[u], l);
    }
}

// Merge chunk partials: o = sum_c o_c e^(m_c-m) / sum_c l_c e^(m_c-m).
__global__ void attn_combine_kernel(AttnArgs a) {
    const int t = blockIdx.x, h = blockIdx.y;
    const int HD = a.head_dim;
    const float *pp = a.part + ((int64_t)t * a.n_heads + h) * a.n_chunks * (HD + 2);
    float m = -INFINITY;
    for (int c = 0; c < a.n_chunks; c++) m = fmaxf(m, pp[c * (HD + 2)]);
    float l = 0.0f;
    for (int c = 0; c < a.n_chunks; c++) {
        const float mc = pp[c * (HD + 2)];
        if (mc != -INFINITY) l = fmaf(pp[c * (HD + 2) + 1], expf(mc - m), l);
    }
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        float o = 0.0f;
        for (int c = 0; c < a.n_chunks; c++) {
            const float mc = pp[c * (HD + 2)];
            if (mc != -INFINITY) o = fmaf(pp[c * (HD + 2) + 2 + d], expf(mc - m), o);
        }
        a.out[(int64_t)t * a.ldo + (int64_t)h * HD + d] = __fdiv_rn(o, l);
    }
}

size_t attention_scratch_bytes(int T, int n_heads, int head_dim, int max_kv_len) {
    int chunks = (max_kv_len + ATT_CH - 1) / ATT_CH;
    if (chunks <= 1) return 0;
    return (size_t)T * n_heads * chunks * (head_dim + 2) * sizeof(float);
}

static size_t attn_smem(int n_heads, int n_kv, int head_dim) {
    const int HW = head_dim >> 1, rw = (HW & 1) ? HW : HW + 1;
    const int qpk = n_heads / n_kv;
    return (size_t)2 * ATT_CH * rw * 4 + (size_t)qpk * head_dim * 4 + (size_t)ATT_WARPS * ATT_CH * 4;
}

int init_noalloc_scratch(vb_ctx *ctx);

int init_attention(vb_ctx *ctx) {
    if (init_noalloc_scratch(ctx)) return VB_ERR_BACKEND;
    VB_CHECK(ctx, cudaFuncSetAttribute(attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
    VB_CHECK(ctx, cudaFuncSetAttribute(attn_segment_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
    return VB_OK;
}

int launch_attention_segments(vb_ctx *ctx, const float *q, int64_t ldq, const uint16_t *k, const uint16_t *v,
                              int n_rows, int n_seg, int T, int n_heads, int n_kv, int head_dim, float *out,
                              int64_t ldo) {
    if (n_seg == 0) return VB_OK;
    if (!q || !k || !v || !out || T <= 0 || T > 32 || n_kv <= 0 || n_heads % n_kv || head_dim % 32 ||
        head_dim > ATT_HD_MAX)
        return set_error(ctx, VB_ERR_INVALID_ARG, "segment attention: bad argument");
    const size_t sm = (size_t)2 * T * head_dim * 4;
    AttnArgs a{};
    a.q = q;
    a.ldq = ldq ? ldq : (int64_t)n_heads * head_dim;
    a.k = k;
    a.v = v;
    a.n_rows = n_rows;
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.head_dim = head_dim;
    a.out = out;
    a.ldo = ldo ? ldo : (int64_t)n_heads * head_dim;
    a.kq_scale = 1.0f / sqrtf((float)head_dim);
    // one warp per (token, query head) row: the rows of a segment and KV
    // group are spread over ceil(T * heads-per-group / ATT_WARPS) CTAs, each
    // staging the group's K/V rows itself (a few KB from L2), so a small
    // batch still fills the GPU
    const int rows = T * (n_heads / n_kv);
    const dim3 grid((unsigned)n_kv, (unsigned)n_seg, (unsigned)((rows + ATT_WARPS - 1) / ATT_WARPS));
    switch (head_dim / 32) {
        case 1: attn_segment_kernel<1><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
        case 2: attn_segment_kernel<2><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
        case 3: attn_segment_kernel<3><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
        case 4: attn_segment_kernel<4><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
        case 5: attn_segment_kernel<5><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
        case 6: attn_segment_kernel<6><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
        case 7: attn_segment_kernel<7><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
        default: attn_segment_kernel<8><<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a, T); break;
    }
    VB_LAUNCH_CHECK(ctx, "attn_segment");
    return VB_OK;
}

// `part` must hold attention_scratch_bytes(); when it is NULL the context
// workspace provides it.
int launch_attention_with(vb_ctx *ctx, const float *q, int64_t ldq, const uint16_t *k, const uint16_t *v,
                          int n_rows, int T, int n_heads, int n_kv, int head_dim, const int32_t *row_start,
                          const int32_t *kv_len, int max_kv_len, float *out, int64_t ldo, float *part) {
    if (T == 0) return VB_OK;
    if (!q || !k || !v || !row_start || !kv_len || !out || n_kv <= 0 || n_heads % n_kv || head_dim % 2 ||
        head_dim > ATT_HD_MAX || max_kv_len <= 0)
        return set_error(ctx, VB_ERR_INVALID_ARG, "attention: bad argument");
    size_t sm = attn_smem(n_heads, n_kv, head_dim);
    if (sm > 160 * 1024) return set_error(ctx, VB_ERR_INVALID_ARG, "attention: head layout too large");
    AttnArgs a;
    a.q = q;
    a.ldq = ldq ? ldq : (int64_t)n_heads * head_dim;
    a.k = k;
    a.v = v;
    a.n_rows = n_rows;
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.head_dim = head_dim;
    a.n_chunks = (max_kv_len + ATT_CH - 1) / ATT_CH;
    a.row_start = row_start;
    a.kv_len = kv_len;
    a.out = out;
    a.ldo = ldo ? ldo : (int64_t)n_heads * head_dim;
    a.part = part;
    a.kq_scale = 1.0f / sqrtf((float)head_dim);
    dim3 grid(a.n_chunks, n_kv, T);
    attn_chunk_kernel<<<grid, ATT_WARPS * 32, sm, ctx->stream>>>(a);
    VB_LAUNCH_CHECK(ctx, "attention_chunks");
    if (a.n_chunks > 1) {
        attn_combine_kernel<<<dim3(T, n_heads), head_dim >= 128 ? 128 : 32, 0, ctx->stream>>>(a);
        VB_LAUNCH_CHECK(ctx, "attention_combine");
    }
    return VB_OK;
}

int launch_attention(vb_ctx *ctx, const float *q, int64_t ldq, const uint16_t *k, const uint16_t *v, int n_rows,
                     int T, int n_heads, int n_kv, int head_dim, const int32_t *row_start, const int32_t *kv_len,
                     int max_kv_len, float *out, int64_t ldo) {
    size_t need = attention_scratch_bytes(T, n_heads, head_dim, max_kv_len);
    float *part = nullptr;
    if (need) {
        int rc = arena_reserve(ctx, ctx->attn_ws, need);
        if (rc) return rc;
        part = (float *)ctx->attn_ws.ptr;
    }
    return launch_attention_with(ctx, q, ldq, k, v, n_rows, T, n_heads, n_kv, head_dim, row_start, kv_len,
                                 max_kv_len, out, ldo, part);
}

// ------------------------------------------------ allocation-free variant
// Scratch for vb_attention_noalloc: the per-chunk (max, sum, partial output)
// records of the flash-decoding split.  It lives in the library image, so
// every device that loads the library holds these bytes until the process
// exits, and no call ever allocates.  Host code must not pass the symbol
// itself to a kernel (on the host it names a stand-in, not device memory):
// init_attention resolves the real device address when a context is
// created, with its device current, and keeps it in the context, so the
// address always belongs to the device context the calls run in.
constexpr size_t NOALLOC_SCRATCH_BYTES = VB_ATTENTION_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) float g_attn_noalloc_scratch[NOALLOC_SCRATCH_BYTES / sizeof(float)];

int init_noalloc_scratch(vb_ctx *ctx) {
    void *p = nullptr;
    VB_CHECK(ctx, cudaGetSymbolAddress(&p, g_attn_noalloc_scratch));
    ctx->attn_noalloc = p;
    return VB_OK;
}

}  // namespace vb

using namespace vb;

extern "C" int vb_attention_noalloc(vb_ctx *ctx, const float *q, const uint16_t *k, const uint16_t *v, int n_rows,
                                    int T, int n_heads, int n_kv_heads, int head_dim, const int32_t *row_start,
                                    const int32_t *kv_len, float *out) {
    if (!ctx) return VB_ERR_INVALID_ARG;
    if (!q || !k || !v || !row_start || !kv_len || !out || n_rows <= 0 || T < 0 || head_dim <= 0 || n_heads <= 0)
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_attention_noalloc: bad argument");
    // same grid as vb_attention: the chunk count comes from n_rows
    const size_t need = attention_scratch_bytes(T, n_heads, head_dim, n_rows);
    if (need > NOALLOC_SCRATCH_BYTES)
        return set_error(ctx, VB_ERR_INVALID_ARG,
                         "vb_attention_noalloc: needs %zu bytes of scratch (T=%d, heads=%d, head_dim=%d, rows=%d); "
                         "the fixed scratch holds %zu bytes -- use vb_attention or fewer rows/tokens per call",
                         need, T, n_heads, head_dim, n_rows, (size_t)NOALLOC_SCRATCH_BYTES);
    float *part = need ? static_cast<float *>(ctx->attn_noalloc) : nullptr;
    if (need && !part) return set_error(ctx, VB_ERR_BACKEND, "vb_attention_noalloc: scratch address unresolved");
    return launch_attention_with(ctx, q, 0, k, v, n_rows, T, n_heads, n_kv_heads, head_dim, row_start, kv_len,
                                 n_rows, out, 0, part);
}
