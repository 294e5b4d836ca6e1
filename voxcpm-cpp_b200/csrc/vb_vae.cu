// vb_vae.cu -- AudioVAE V2 decoder (latent patches -> 48 kHz PCM) as CUDA
// kernels, streaming over a batch of independent utterances.
//
// Reference: the streaming decoder graph of src/audio_vae_stream.c:184-619
// (per-layer history caches, vcpm_vae_stream_create/reset/decode) and the
// layer helpers of src/audio_vae_v2.c (causal depthwise / pointwise conv
// :214-407, transposed conv with causal trim :409-441, Snake :483-503,
// residual unit :567-636, block table :40-43).
//
// Layout: activations are time-major [stream][time][channels] in F32, so a
// pointwise conv is a GEMM with M = streams x time and K = input channels,
// and a transposed conv of stride s (kernel 2s) is one GEMM as well: output
// times q*s .. q*s+s-1 of all channels form one row of s*Co values, computed
// from the concatenated input rows [x(q-1) | x(q)] (x(-1) = the history
// cache) against a repacked weight [2*Ci][s*Co].  The GEMM is an fp32 SIMT
// kernel, or for the wide layers the tcgen05 GEMM with both operands split
// into tf32 hi/lo (three products, fp32-class accuracy; a single tf32 or
// bf16 product would move PCM by ~1e-3), with the bias, residual skip,
// sr_cond scale/bias and the next layer's Snake fused into its epilogue.
// Depthwise k7 convs and the final k7 -> tanh conv are bandwidth-bound
// direct kernels that also roll their history caches (double-buffered, so
// no launch reads a cache row that the same launch rewrites).
#include <algorithm>
#include <cstring>
#include <vector>

#include "vb_common.cuh"
#include "vb_kernels.cuh"

using namespace vb;

namespace {

constexpr int VAE_DIL[3] = {1, 3, 9};

// snake(x, a) = x + sin(a*x)^2 / a, one fp32 op at a time as ggml's
// mul / sin / sqr / div / add nodes (src/audio_vae_v2.c:483-503).
__device__ __forceinline__ float snake_f(float x, float a) {
    const float t = __fmul_rn(x, a);
    const float st = sinf(t);
    const float sq = __fmul_rn(st, st);
    return __fadd_rn(x, __fdiv_rn(sq, a));
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }

// tf32 of x with round-to-nearest-even (fp32 storage, low 13 mantissa bits
// clear, as the tensor core reads it); finite inputs.
__host__ __device__ __forceinline__ uint32_t tf32_bits(uint32_t u) {
    if ((u & 0x7f800000u) == 0x7f800000u) return u;
    u += 0xfffu + ((u >> 13) & 1u);
    return u & 0xffffe000u;
}

// x = hi + lo: hi = tf32(x), lo = tf32(x - hi) (the difference is exact).
__device__ __forceinline__ void split4(float4 v, float *hi, float *lo) {
    const float x[4] = {v.x, v.y, v.z, v.w};
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        h[e] = __uint_as_float(tf32_bits(__float_as_uint(x[e])));
        l[e] = __uint_as_float(tf32_bits(__float_as_uint(__fsub_rn(x[e], h[e]))));
    }
    st4(hi, make_float4(h[0], h[1], h[2], h[3]));
    st4(lo, make_float4(l[0], l[1], l[2], l[3]));
}

// ----------------------------------------------------------------- GEMM
struct VaeGemm {
    const float *A;       // [M][Ka] rows
    int Ka;
    const float *prev;    // non-null: K = 2*Ka, k < Ka reads the previous row (prev[stream] for a stream's first row)
    int T_in;             // rows per stream (for the previous-row rule)
    const float *B;       // [K][N]
    int M, N, K;
    const float *bias;    // [Cb], index n % Cb
    int Cb;
    const float *skip;    // [M][N] residual added after the bias (may alias out_h)
    float *out_h;         // [M][N] value
    float *out_x;         // [M][N] next layer's input: snake(alpha)(sr(value))
    const float *alpha, *sr_scale, *sr_bias;   // [Cb] each, optional
};

constexpr int G_BK = 8, G_THREADS = 256;

// Epilogue of four consecutive values (n % 4 == 0, N % 4 == 0, Cb % 4 == 0):
// bias, skip, then the outputs; every op one fp32 rounding, as ggml's nodes.
__device__ __forceinline__ void gemm_out4(const VaeGemm &g, int64_t m, int n, float4 acc) {
    const int c = n % g.Cb;
    float v[4] = {acc.x, acc.y, acc.z, acc.w};
    if (g.bias) {
        const float4 b = ld4(g.bias + c);
        v[0] = __fadd_rn(v[0], b.x); v[1] = __fadd_rn(v[1], b.y);
        v[2] = __fadd_rn(v[2], b.z); v[3] = __fadd_rn(v[3], b.w);
    }
    const int64_t at = m * g.N + n;
    if (g.skip) {
        const float4 k = ld4(g.skip + at);
        v[0] = __fadd_rn(k.x, v[0]); v[1] = __fadd_rn(k.y, v[1]);
        v[2] = __fadd_rn(k.z, v[2]); v[3] = __fadd_rn(k.w, v[3]);
    }
    if (g.out_h) st4(g.out_h + at, make_float4(v[0], v[1], v[2], v[3]));
    if (g.out_x) {
        if (g.sr_scale) {
            const float4 a = ld4(g.sr_scale + c), b = ld4(g.sr_bias + c);
            v[0] = __fadd_rn(__fmul_rn(v[0], a.x), b.x); v[1] = __fadd_rn(__fmul_rn(v[1], a.y), b.y);
            v[2] = __fadd_rn(__fmul_rn(v[2], a.z), b.z); v[3] = __fadd_rn(__fmul_rn(v[3], a.w), b.w);
        }
        if (g.alpha) {
            const float4 a = ld4(g.alpha + c);
            v[0] = snake_f(v[0], a.x); v[1] = snake_f(v[1], a.y);
            v[2] = snake_f(v[2], a.z); v[3] = snake_f(v[3], a.w);
        }
        st4(g.out_x + at, make_float4(v[0], v[1], v[2], v[3]));
    }
}

// The two source rows of logical A row m: columns k < split come from `lo`,
// the rest from `hi` (one row when there is no previous-row part).
struct ARow {
    const float *lo, *hi;
    int split;
    bool valid;
};

__device__ __forceinline__ ARow gemm_a_row(const VaeGemm &g, int64_t m) {
    ARow r;
    r.valid = m < g.M;
    const float *cur = g.A + (r.valid ? m : 0) * g.Ka;
    if (!g.prev) {
        r.lo = r.hi = cur;
        r.split = g.K;
    } else {
        const int64_t t = r.valid ? m % g.T_in : 0;
        r.lo = t ? cur - g.Ka : g.prev + (r.valid ? m / g.T_in : 0) * g.Ka;
        r.hi = cur - g.Ka;      // indexed from k = Ka
        r.split = g.Ka;
    }
    return r;
}

// A float4 of row r at columns k..k+3 (k % 4 == 0).
__device__ __forceinline__ float4 gemm_load_a(const VaeGemm &g, const ARow &r, int k) {
    if (!r.valid || k >= g.K) return make_float4(0.f, 0.f, 0.f, 0.f);
    return ld4((k < r.split ? r.lo : r.hi) + k);
}

// C[M][N] = A[M][K] . B[K][N] with the fused epilogue.  BM x BN tile, 256
// threads, TM x TN outputs per thread: rows ty*TM.., columns in TN/4 groups
// of four at g*(BN/G) + tx*4, so that a quarter-warp's shared-memory reads
// and global stores of B / C cover one contiguous span.  A is staged
// transposed in shared memory; both operands are double-buffered through
// registers.  Each output accumulates over k in order with fmaf.
template <int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__(G_THREADS, 2) vae_gemm_kernel(const VaeGemm g) {
    constexpr int TX = BN / (TN / 4) / 4;     // threads along N per column group
    constexpr int G = TN / 4;                 // column groups per thread
    static_assert((BM / TM) * TX == G_THREADS, "thread tiling");
    static_assert(TM % 4 == 0 && TN % 4 == 0, "vector widths");
    __shared__ __align__(16) float As[2][G_BK][BM + 4];
    __shared__ __align__(16) float Bs[2][G_BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const int64_t m0 = (int64_t)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    // loaders: A row tid/2, k quad (tid%2)*4 (BM*2 threads); B k-row
    // tid/(BN/4), column quad (BN*2 threads)
    const bool aload = tid < BM * 2;
    const int ar = (tid >> 1) % BM, ak = (tid & 1) * 4;
    const bool bload = tid < 2 * BN;
    const int bk = (tid / (BN / 4)) % G_BK, bn = (tid % (BN / 4)) * 4;

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0.f;

    auto load_b = [&](int k0) -> float4 {
        const int k = k0 + bk, n = n0 + bn;
        if (!bload || k >= g.K || n >= g.N) return make_float4(0.f, 0.f, 0.f, 0.f);
        return ld4(g.B + (int64_t)k * g.N + n);
    };
    const ARow arow = gemm_a_row(g, m0 + ar);
    float4 ra = aload ? gemm_load_a(g, arow, ak) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 rb = load_b(0);
    const int nk = (g.K + G_BK - 1) / G_BK;
    int buf = 0;
    if (aload) {
        As[0][ak + 0][ar] = ra.x; As[0][ak + 1][ar] = ra.y; As[0][ak + 2][ar] = ra.z; As[0][ak + 3][ar] = ra.w;
    }
    if (bload) st4(&Bs[0][bk][bn], rb);
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        const bool more = kt + 1 < nk;
        if (more) {
            if (aload) ra = gemm_load_a(g, arow, (kt + 1) * G_BK + ak);
            rb = load_b((kt + 1) * G_BK);
        }
#pragma unroll
        for (int k = 0; k < G_BK; k++) {
            float a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < TM; i += 4) {
                const float4 v = *reinterpret_cast<const float4 *>(&As[buf][k][ty * TM + i]);
                a[i] = v.x; a[i + 1] = v.y; a[i + 2] = v.z; a[i + 3] = v.w;
            }
#pragma unroll
            for (int q = 0; q < G; q++) {
                const float4 v = *reinterpret_cast<const float4 *>(&Bs[buf][k][q * (BN / G) + tx * 4]);
                b[4 * q] = v.x; b[4 * q + 1] = v.y; b[4 * q + 2] = v.z; b[4 * q + 3] = v.w;
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            const int nb = buf ^ 1;
            if (aload) {
                As[nb][ak + 0][ar] = ra.x; As[nb][ak + 1][ar] = ra.y; As[nb][ak + 2][ar] = ra.z; As[nb][ak + 3][ar] = ra.w;
            }
            if (bload) st4(&Bs[nb][bk][bn], rb);
            __syncthreads();
            buf = nb;
        }
    }
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int64_t m = m0 + ty * TM + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int q = 0; q < G; q++) {
            const int n = n0 + q * (BN / G) + tx * 4;
            if (n < g.N)
                gemm_out4(g, m, n, make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]));
        }
    }
}

// ------------------------------------------------------ depthwise conv k7
// y[b][t][c] = snake(alpha)(sum_j w[j][c] * comb[t + j*d][c] + bias[c]),
// comb = [history (6d rows); x (T rows)]; rows T .. T+6d-1 of the grid
// write the new history (the last 6d rows of comb) into cnew.
__global__ void vae_dw7_kernel(const float *__restrict__ x, const float *__restrict__ cold, float *__restrict__ cnew,
                               const float *__restrict__ w, const float *__restrict__ bias,
                               const float *__restrict__ alpha, float *__restrict__ y, float *__restrict__ ylo, int T,
                               int C, int d) {
    const int C4 = C / 4, L = 6 * d, b = blockIdx.y;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)(T + L) * C4) return;
    const int row = (int)(idx / C4), c = (int)(idx % C4) * 4;
    const float *xb = x + (int64_t)b * T * C;
    const float *hb = cold + (int64_t)b * L * C;
    auto comb = [&](int i) -> const float * { return i < L ? hb + (int64_t)i * C : xb + (int64_t)(i - L) * C; };
    if (row >= T) {
        const int r = row - T;
        st4(cnew + ((int64_t)b * L + r) * C + c, ld4(comb(T + r) + c));
        return;
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 7; j++) {
        const float4 v = ld4(comb(row + j * d) + c), k = ld4(w + j * C + c);
        acc.x = fmaf(k.x, v.x, acc.x);
        acc.y = fmaf(k.y, v.y, acc.y);
        acc.z = fmaf(k.z, v.z, acc.z);
        acc.w = fmaf(k.w, v.w, acc.w);
    }
    if (bias) {
        const float4 bb = ld4(bias + c);
        acc.x = __fadd_rn(acc.x, bb.x); acc.y = __fadd_rn(acc.y, bb.y);
        acc.z = __fadd_rn(acc.z, bb.z); acc.w = __fadd_rn(acc.w, bb.w);
    }
    if (alpha) {
        const float4 a = ld4(alpha + c);
        acc.x = snake_f(acc.x, a.x); acc.y = snake_f(acc.y, a.y);
        acc.z = snake_f(acc.z, a.z); acc.w = snake_f(acc.w, a.w);
    }
    const int64_t at = ((int64_t)b * T + row) * C + c;
    if (ylo) split4(acc, y + at, ylo + at);     // tf32 hi/lo operand of the next GEMM
    else st4(y + at, acc);
}

// The transposed conv's GEMM operand as tf32 hi/lo rows [x(q-1) | x(q)] of
// 2C values (x(-1) = the stream's history row).
__global__ void vae_split_prev_kernel(const float *__restrict__ x, const float *__restrict__ hist,
                                      float *__restrict__ ah, float *__restrict__ al, int64_t M, int T, int C) {
    const int C4 = C / 4;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= M * 2 * C4) return;
    const int64_t m = idx / (2 * C4);
    const int q = (int)(idx % (2 * C4)), half = q / C4, c = (q % C4) * 4;
    const int64_t t = m % T;
    const float *src = half ? x + m * C : (t ? x + (m - 1) * C : hist + (m / T) * C);
    const int64_t at = m * 2 * C + (int64_t)half * C + c;
    split4(ld4(src + c), ah + at, al + at);
}

// ------------------------------------------- output conv k7, C -> 1, tanh
// audio[b][t] = tanh(sum_{i,j} w[i][j] * comb[t + j][i] + bias), summed
// channel-major / tap-minor (im2col order).  A CTA stages the OUT7_T + 6
// history/input rows it needs in shared memory (row stride C + 1: the
// per-thread row reads then hit distinct banks) and each thread computes
// one sample; the CTA holding the stream's last samples also rolls the
// history (the last 6 rows of comb).
constexpr int OUT7_T = 128;

__global__ void __launch_bounds__(OUT7_T) vae_out7_kernel(const float *__restrict__ x, const float *__restrict__ cold,
                                                           float *__restrict__ cnew, const float *__restrict__ w,
                                                           const float *__restrict__ bias, float *__restrict__ audio,
                                                           int T, int C) {
    extern __shared__ float o7[];          // [OUT7_T + 6][C + 1], then w [C][7]
    const int L = 6, b = blockIdx.y, t0 = blockIdx.x * OUT7_T;
    const int CS = C + 1;
    float *ws = o7 + (OUT7_T + L) * CS;
    const float *xb = x + (int64_t)b * T * C;
    const float *hb = cold + (int64_t)b * L * C;
    auto comb = [&](int i) -> const float * { return i < L ? hb + (int64_t)i * C : xb + (int64_t)(i - L) * C; };
    const int rows = min(OUT7_T + L, T + L - t0);
    for (int e = threadIdx.x; e < rows * C; e += OUT7_T) {
        const int r = e / C, c = e - r * C;
        o7[r * CS + c] = comb(t0 + r)[c];
    }
    for (int e = threadIdx.x; e < C * 7; e += OUT7_T) ws[e] = w[e];
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t < T) {
        float acc = 0.f;
        for (int i = 0; i < C; i++)
#pragma unroll
            for (int j = 0; j < 7; j++) acc = fmaf(ws[i * 7 + j], o7[(threadIdx.x + j) * CS + i], acc);
        float v = acc;
        if (bias) v = __fadd_rn(v, bias[0]);
        audio[(int64_t)b * T + t] = tanhf(v);
    }
    if (t0 + OUT7_T >= T) {        // this CTA covers the stream's end: new history = comb[T .. T+5]
        for (int e = threadIdx.x; e < L * C; e += OUT7_T) {
            const int r = e / C, c = e - r * C;
            cnew[((int64_t)b * L + r) * C + c] = comb(T + r)[c];
        }
    }
}

// ------------------------------------------------------------ host side
float host_h2f(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

}  // namespace

struct VaeResUnit {
    float *alpha0 = nullptr, *dw_w = nullptr, *dw_b = nullptr, *alpha2 = nullptr, *pw_w = nullptr, *pw_b = nullptr;
    Tf32Weight pw_t;              // tensor-core operand of pw_w ([Co][Co], hi/lo), if used
};
struct VaeBlock {
    int ci = 0, co = 0, s = 0;
    float *sr_scale = nullptr, *sr_bias = nullptr, *alpha = nullptr, *up_w = nullptr, *up_b = nullptr;
    Tf32Weight up_t;              // [s*Co][2*Ci] hi/lo, if used
    VaeResUnit res[3];
};

struct vb_vae_s {
    vb_vae_config cfg{};
    bool tf32 = true;             // tensor-core path for the wide convs (VB_VAE_TF32=0: fp32 SIMT everywhere)
    float *in_dw_w = nullptr, *in_dw_b = nullptr, *in_pw_w = nullptr, *in_pw_b = nullptr;
    Tf32Weight in_pw_t;           // [D][latent] hi/lo, if used
    VaeBlock blk[6];
    float *out_alpha = nullptr, *out_w = nullptr, *out_b = nullptr;
    std::vector<void *> allocs;
    size_t device_bytes = 0;
};

struct vb_vae_stream_s {
    vb_vae vae = nullptr;
    int n = 0;                    // streams (utterances) decoded in lockstep
    int n0 = 0;                   // streams at creation (the caches' row capacity)
    std::vector<int32_t> utt;     // utterance index of each current row
    int32_t *map_dev = nullptr;   // [n0] row map of a retire
    float *tmp = nullptr;         // gather scratch of a retire (largest cache)
    int patch_size = 0;
    int parity = 0;               // which half of each double-buffered history is current
    float *cache_in[2] = {};      // [n][6][latent]
    float *cache_up[6] = {};      // [n][Ci]
    float *cache_res[6][3][2] = {};   // [n][6d][Co]
    float *cache_out[2] = {};     // [n][6][C_last]
    std::vector<void *> allocs;
    size_t state_bytes = 0;
    float *work = nullptr;        // activations: X0, XA, XB, TB, H, then the tf32 operand AH, AL (2x each)
    size_t work_floats = 0;       // per buffer
    int work_T = 0;               // latent frames the buffers hold
};

namespace {

int vae_upsample(const vb_vae_config &c) {
    int f = 1;
    for (int i = 0; i < 6; i++) f *= c.rates[i];
    return f;
}

// Copies a host tensor of `n` elements (F32, or F16 when `f16`) to F32.
void to_f32(const void *src, bool f16, size_t n, std::vector<float> &out) {
    out.resize(n);
    if (f16) {
        const uint16_t *h = static_cast<const uint16_t *>(src);
        for (size_t i = 0; i < n; i++) out[i] = host_h2f(h[i]);
    } else {
        memcpy(out.data(), src, n * sizeof(float));
    }
}

float host_tf32(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    u = tf32_bits(u);
    float r;
    memcpy(&r, &u, 4);
    return r;
}

// Wide convs (N >= 128 output values per row, K >= 256 and a multiple of
// 32) run on the tensor cores as three tf32 products; the rest on the SIMT
// kernel (measured on B200: below K = 256 the tensor-core tiles wait on
// their epilogue and the SIMT kernel is as fast).
bool use_tf32(const vb_vae_s *v, int N, int K) { return v->tf32 && N >= 128 && K >= 256 && K % 32 == 0; }

int upload(vb_ctx *ctx, vb_vae v, const std::vector<float> &h, float **dst);

// K-major [N][K] weight -> tf32 hi/lo device copies.
int upload_tf32(vb_ctx *ctx, vb_vae v, const std::vector<float> &wk, int N, int K, Tf32Weight &t) {
    std::vector<float> hi(wk.size()), lo(wk.size());
    for (size_t i = 0; i < wk.size(); i++) {
        hi[i] = host_tf32(wk[i]);
        lo[i] = host_tf32(wk[i] - hi[i]);
    }
    t.N = N;
    t.K = K;
    int rc = upload(ctx, v, hi, &t.hi);
    if (!rc) rc = upload(ctx, v, lo, &t.lo);
    return rc;
}

int upload(vb_ctx *ctx, vb_vae v, const std::vector<float> &h, float **dst) {
    *dst = nullptr;
    if (h.empty()) return VB_OK;
    void *p = nullptr;
    if (cudaMalloc(&p, h.size() * sizeof(float)) != cudaSuccess)
        return set_error(ctx, VB_ERR_OOM, "vb_vae_create: device allocation of %zu bytes failed", h.size() * 4);
    v->allocs.push_back(p);
    v->device_bytes += h.size() * sizeof(float);
    VB_CHECK(ctx, cudaMemcpy(p, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
    *dst = static_cast<float *>(p);
    return VB_OK;
}

template <int BM, int BN, int TM, int TN>
int launch_gemm_tile(vb_ctx *ctx, const VaeGemm &g) {
    dim3 grid((unsigned)((g.M + BM - 1) / BM), (unsigned)((g.N + BN - 1) / BN));
    vae_gemm_kernel<BM, BN, TM, TN><<<grid, G_THREADS, 0, ctx->stream>>>(g);
    VB_LAUNCH_CHECK(ctx, "vae_gemm");
    return VB_OK;
}

// Widest N tile the shape fills; 64-row tiles when 128-row ones would give
// fewer than two CTAs per SM.
int launch_vae_gemm(vb_ctx *ctx, const VaeGemm &g) {
    if (g.M <= 0) return VB_OK;
    const int64_t bn = g.N >= 128 ? 128 : (g.N >= 64 ? 64 : 32);
    const int64_t tiles128 = (g.M + 127) / 128 * ((g.N + bn - 1) / bn);
    const bool small = tiles128 < 2 * (int64_t)ctx->sm_count;
    if (bn == 128) return small ? launch_gemm_tile<64, 128, 4, 8>(ctx, g) : launch_gemm_tile<128, 128, 8, 8>(ctx, g);
    if (bn == 64) return small ? launch_gemm_tile<64, 64, 4, 4>(ctx, g) : launch_gemm_tile<128, 64, 8, 4>(ctx, g);
    return launch_gemm_tile<128, 32, 4, 4>(ctx, g);
}

// y_lo non-null: y and y_lo receive the tf32 hi/lo split of the output.
int launch_dw7(vb_ctx *ctx, const float *x, const float *cold, float *cnew, const float *w, const float *bias,
               const float *alpha, float *y, float *y_lo, int n, int T, int C, int d) {
    const int64_t items = (int64_t)(T + 6 * d) * (C / 4);
    dim3 grid((unsigned)((items + 255) / 256), (unsigned)n);
    vae_dw7_kernel<<<grid, 256, 0, ctx->stream>>>(x, cold, cnew, w, bias, alpha, y, y_lo, T, C, d);
    VB_LAUNCH_CHECK(ctx, "vae_dw7");
    return VB_OK;
}

}  // namespace

extern "C" int vb_vae_create(vb_ctx *ctx, const vb_vae_config *cfg, const void *const *t, vb_vae *out) {
    if (!ctx || !cfg || !t || !out) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    const vb_vae_config &c = *cfg;
    if (c.latent_dim <= 0 || c.latent_dim % 4 || c.decoder_dim <= 0 || c.decoder_dim % 256)
        return set_error(ctx, VB_ERR_INVALID_ARG,
                         "vb_vae_create: latent_dim must be a multiple of 4 and decoder_dim of 256");
    for (int i = 0; i < 6; i++)
        if (c.rates[i] <= 0 || c.rates[i] > 64) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_create: bad rate");
    if (c.weight_type != VB_TYPE_F32 && c.weight_type != VB_TYPE_F16)
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_create: conv weights must be F32 or F16");
    if (!t[VB_VAE_IN_DW_W] || !t[VB_VAE_IN_PW_W] || !t[VB_VAE_OUT_W])
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_create: missing model.0 / model.1 / model.9 weight");
    for (int b = 0; b < 6; b++) {
        const int base = VB_VAE_BLOCK0 + b * VB_VAE_BLOCK_SLOTS;
        if (!t[base + VB_VAE_B_UP_W])
            return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_create: missing upsample weight of block %d", b);
        if (!t[base + VB_VAE_B_SR_SCALE] != !t[base + VB_VAE_B_SR_BIAS])
            return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_create: sr_cond scale and bias go together");
        for (int u = 0; u < 3; u++) {
            const int rb = base + VB_VAE_B_RES0 + u * VB_VAE_RES_SLOTS;
            if (!t[rb + VB_VAE_R_DW_W] || !t[rb + VB_VAE_R_PW_W])
                return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_create: missing residual conv of block %d", b);
        }
    }
    if (fault_injected("alloc")) return set_error(ctx, VB_ERR_OOM, "vb_vae_create: injected allocation fault");
    VB_CHECK(ctx, cudaSetDevice(ctx->device));
    vb_vae v = new vb_vae_s();
    v->cfg = c;
    {
        const char *e = getenv("VB_VAE_TF32");
        v->tf32 = !(e && e[0] == '0');
    }
    const bool f16 = c.weight_type == VB_TYPE_F16;
    const int L = c.latent_dim, D = c.decoder_dim;
    std::vector<float> a, r;
    auto vec = [&](const void *p, size_t n, float **dst) -> int {   // per-channel F32 vectors
        if (!p) { *dst = nullptr; return VB_OK; }
        to_f32(p, false, n, a);
        return upload(ctx, v, a, dst);
    };
    // depthwise [C][7] -> [7][C]
    auto dw = [&](const void *p, int C, float **dst) -> int {
        to_f32(p, f16, (size_t)C * 7, a);
        r.assign((size_t)C * 7, 0.f);
        for (int ch = 0; ch < C; ch++)
            for (int j = 0; j < 7; j++) r[(size_t)j * C + ch] = a[(size_t)ch * 7 + j];
        return upload(ctx, v, r, dst);
    };
    // pointwise [Co][Ci] -> B operand [Ci][Co] (SIMT), and the [Co][Ci]
    // tf32 hi/lo pair when the layer runs on the tensor cores
    auto pw = [&](const void *p, int ci, int co, float **dst, Tf32Weight *tw) -> int {
        to_f32(p, f16, (size_t)ci * co, a);
        r.assign((size_t)ci * co, 0.f);
        for (int o = 0; o < co; o++)
            for (int i = 0; i < ci; i++) r[(size_t)i * co + o] = a[(size_t)o * ci + i];
        int rc2 = upload(ctx, v, r, dst);
        if (!rc2 && use_tf32(v, co, ci)) rc2 = upload_tf32(ctx, v, a, co, ci, *tw);
        return rc2;
    };
    int rc = VB_OK;
    if (!rc) rc = dw(t[VB_VAE_IN_DW_W], L, &v->in_dw_w);
    if (!rc) rc = vec(t[VB_VAE_IN_DW_B], L, &v->in_dw_b);
    if (!rc) rc = pw(t[VB_VAE_IN_PW_W], L, D, &v->in_pw_w, &v->in_pw_t);
    if (!rc) rc = vec(t[VB_VAE_IN_PW_B], D, &v->in_pw_b);
    for (int b = 0; b < 6 && !rc; b++) {
        VaeBlock &B = v->blk[b];
        B.ci = D >> b;
        B.co = D >> (b + 1);
        B.s = c.rates[b];
        const int base = VB_VAE_BLOCK0 + b * VB_VAE_BLOCK_SLOTS, ci = B.ci, co = B.co, s = B.s;
        rc = vec(t[base + VB_VAE_B_SR_SCALE], ci, &B.sr_scale);
        if (!rc) rc = vec(t[base + VB_VAE_B_SR_BIAS], ci, &B.sr_bias);
        if (!rc) rc = vec(t[base + VB_VAE_B_ALPHA], ci, &B.alpha);
        if (!rc) rc = vec(t[base + VB_VAE_B_UP_B], co, &B.up_b);
        if (!rc) {
            // [Ci][Co][2s] -> [2*Ci][s*Co]: rows 0..Ci-1 take the previous
            // input through taps s..2s-1, rows Ci.. the current one through 0..s-1
            to_f32(t[base + VB_VAE_B_UP_W], f16, (size_t)ci * co * 2 * s, a);
            r.assign((size_t)2 * ci * s * co, 0.f);
            for (int i = 0; i < ci; i++)
                for (int o = 0; o < co; o++)
                    for (int q = 0; q < s; q++) {
                        const size_t src = ((size_t)i * co + o) * 2 * s;
                        r[(size_t)i * s * co + (size_t)q * co + o] = a[src + s + q];
                        r[(size_t)(ci + i) * s * co + (size_t)q * co + o] = a[src + q];
                    }
            rc = upload(ctx, v, r, &B.up_w);
            if (!rc && use_tf32(v, s * co, 2 * ci)) {
                // K-major [s*Co][2*Ci]: row q*Co + o, previous-row taps then current-row taps
                std::vector<float> wk((size_t)s * co * 2 * ci);
                for (int q = 0; q < s; q++)
                    for (int o = 0; o < co; o++) {
                        float *row = wk.data() + ((size_t)q * co + o) * 2 * ci;
                        for (int i = 0; i < ci; i++) {
                            const size_t src = ((size_t)i * co + o) * 2 * s;
                            row[i] = a[src + s + q];
                            row[ci + i] = a[src + q];
                        }
                    }
                rc = upload_tf32(ctx, v, wk, s * co, 2 * ci, B.up_t);
            }
        }
        for (int u = 0; u < 3 && !rc; u++) {
            const int rb = base + VB_VAE_B_RES0 + u * VB_VAE_RES_SLOTS;
            VaeResUnit &R = B.res[u];
            rc = vec(t[rb + VB_VAE_R_ALPHA0], co, &R.alpha0);
            if (!rc) rc = dw(t[rb + VB_VAE_R_DW_W], co, &R.dw_w);
            if (!rc) rc = vec(t[rb + VB_VAE_R_DW_B], co, &R.dw_b);
            if (!rc) rc = vec(t[rb + VB_VAE_R_ALPHA2], co, &R.alpha2);
            if (!rc) rc = pw(t[rb + VB_VAE_R_PW_W], co, co, &R.pw_w, &R.pw_t);
            if (!rc) rc = vec(t[rb + VB_VAE_R_PW_B], co, &R.pw_b);
        }
    }
    const int cl = D >> 6;
    if (!rc) rc = vec(t[VB_VAE_OUT_ALPHA], cl, &v->out_alpha);
    if (!rc) {
        to_f32(t[VB_VAE_OUT_W], f16, (size_t)cl * 7, a);
        rc = upload(ctx, v, a, &v->out_w);
    }
    if (!rc) rc = vec(t[VB_VAE_OUT_B], 1, &v->out_b);
    if (rc) {
        vb_vae_destroy(ctx, v);
        return rc;
    }
    *out = v;
    return VB_OK;
}

extern "C" void vb_vae_destroy(vb_ctx *ctx, vb_vae v) {
    if (!v) return;
    if (ctx) cudaStreamSynchronize(ctx->stream);
    for (void *p : v->allocs) cudaFree(p);
    delete v;
}

extern "C" size_t vb_vae_device_bytes(vb_vae v) { return v ? v->device_bytes : 0; }

extern "C" int vb_vae_stream_create(vb_ctx *ctx, vb_vae v, int n_streams, int patch_size, vb_vae_stream *out) {
    if (!ctx || !v || !out || n_streams <= 0 || patch_size <= 0) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    if (fault_injected("alloc")) return set_error(ctx, VB_ERR_OOM, "vb_vae_stream_create: injected allocation fault");
    vb_vae_stream s = new vb_vae_stream_s();
    s->vae = v;
    s->n = s->n0 = n_streams;
    s->patch_size = patch_size;
    const vb_vae_config &c = v->cfg;
    const int D = c.decoder_dim;
    auto alloc = [&](size_t floats, float **dst) -> bool {
        void *p = nullptr;
        if (cudaMalloc(&p, floats * sizeof(float)) != cudaSuccess) return false;
        s->allocs.push_back(p);
        s->state_bytes += floats * sizeof(float);
        *dst = static_cast<float *>(p);
        return true;
    };
    bool ok = true;
    for (int h = 0; h < 2; h++) ok = ok && alloc((size_t)n_streams * 6 * c.latent_dim, &s->cache_in[h]);
    for (int b = 0; b < 6 && ok; b++) {
        ok = alloc((size_t)n_streams * (D >> b), &s->cache_up[b]);
        for (int u = 0; u < 3 && ok; u++)
            for (int h = 0; h < 2 && ok; h++)
                ok = alloc((size_t)n_streams * 6 * VAE_DIL[u] * (D >> (b + 1)), &s->cache_res[b][u][h]);
    }
    for (int h = 0; h < 2 && ok; h++) ok = alloc((size_t)n_streams * 6 * (D >> 6), &s->cache_out[h]);
    if (ok) {
        // retire scratch: the row map and one gather buffer of the largest cache
        size_t big = (size_t)6 * c.latent_dim;
        for (int b = 0; b < 6; b++) big = std::max(big, (size_t)6 * VAE_DIL[2] * (D >> (b + 1)));
        big = std::max(big, (size_t)D);
        void *m = nullptr, *t = nullptr;
        ok = cudaMalloc(&m, (size_t)n_streams * 4) == cudaSuccess;
        if (ok) s->allocs.push_back(m);
        ok = ok && cudaMalloc(&t, big * n_streams * sizeof(float)) == cudaSuccess;
        if (ok) s->allocs.push_back(t);
        s->map_dev = static_cast<int32_t *>(m);
        s->tmp = static_cast<float *>(t);
    }
    if (!ok) {
        vb_vae_stream_destroy(ctx, s);
        return set_error(ctx, VB_ERR_OOM, "vb_vae_stream_create: history allocation failed");
    }
    const int rc = vb_vae_stream_reset(ctx, s);
    if (rc) {
        vb_vae_stream_destroy(ctx, s);
        return rc;
    }
    *out = s;
    return VB_OK;
}

extern "C" int vb_vae_stream_reset(vb_ctx *ctx, vb_vae_stream s) {
    if (!ctx || !s) return VB_ERR_INVALID_ARG;
    // every stream of the creation, in utterance order, from zero history
    s->n = s->n0;
    s->utt.resize(s->n0);
    for (int i = 0; i < s->n0; i++) s->utt[i] = i;
    const vb_vae_config &c = s->vae->cfg;
    const int D = c.decoder_dim, n = s->n;
    for (int h = 0; h < 2; h++) {
        VB_CHECK(ctx, cudaMemsetAsync(s->cache_in[h], 0, sizeof(float) * n * 6 * c.latent_dim, ctx->stream));
        VB_CHECK(ctx, cudaMemsetAsync(s->cache_out[h], 0, sizeof(float) * n * 6 * (D >> 6), ctx->stream));
    }
    for (int b = 0; b < 6; b++) {
        VB_CHECK(ctx, cudaMemsetAsync(s->cache_up[b], 0, sizeof(float) * n * (D >> b), ctx->stream));
        for (int u = 0; u < 3; u++)
            for (int h = 0; h < 2; h++)
                VB_CHECK(ctx, cudaMemsetAsync(s->cache_res[b][u][h], 0,
                                              sizeof(float) * n * 6 * VAE_DIL[u] * (D >> (b + 1)), ctx->stream));
    }
    s->parity = 0;
    return VB_OK;
}

namespace vb {
__global__ void vae_gather_rows_kernel(const float *src, float *dst, const int32_t *map, int rows, int64_t width) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * width) return;
    const int64_t r = i / width, c = i % width;
    dst[i] = src[(int64_t)map[r] * width + c];
}
}  // namespace vb

extern "C" int vb_vae_stream_retire(vb_ctx *ctx, vb_vae_stream s, int n, const int32_t *utterances) {
    if (!ctx || !s || n < 0 || (n > 0 && !utterances)) return VB_ERR_INVALID_ARG;
    std::vector<char> drop(s->n, 0);
    bool any = false;
    for (int i = 0; i < n; i++)
        for (int r = 0; r < s->n; r++)
            if (s->utt[r] == utterances[i] && !drop[r]) {
                drop[r] = 1;
                any = true;
            }
    if (!any) return VB_OK;
    std::vector<int32_t> map, utt;
    for (int r = 0; r < s->n; r++)
        if (!drop[r]) {
            map.push_back(r);
            utt.push_back(s->utt[r]);
        }
    const int nk = (int)map.size();
    if (nk > 0) {
        const vb_vae_config &c = s->vae->cfg;
        const int D = c.decoder_dim;
        std::vector<std::pair<float *, int64_t>> bufs;   // cache, floats per stream
        for (int h = 0; h < 2; h++) {
            bufs.push_back({s->cache_in[h], (int64_t)6 * c.latent_dim});
            bufs.push_back({s->cache_out[h], (int64_t)6 * (D >> 6)});
        }
        for (int b = 0; b < 6; b++) {
            bufs.push_back({s->cache_up[b], (int64_t)(D >> b)});
            for (int u = 0; u < 3; u++)
                for (int h = 0; h < 2; h++) bufs.push_back({s->cache_res[b][u][h], (int64_t)6 * VAE_DIL[u] * (D >> (b + 1))});
        }
        VB_CHECK(ctx, cudaMemcpyAsync(s->map_dev, map.data(), (size_t)nk * 4, cudaMemcpyHostToDevice, ctx->stream));
        for (auto &bw : bufs) {
            const int64_t total = (int64_t)nk * bw.second;
            vae_gather_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, ctx->stream>>>(bw.first, s->tmp, s->map_dev,
                                                                                           nk, bw.second);
            VB_LAUNCH_CHECK(ctx, "vae_gather_rows");
            VB_CHECK(ctx, cudaMemcpyAsync(bw.first, s->tmp, (size_t)total * 4, cudaMemcpyDeviceToDevice, ctx->stream));
        }
    }
    // the host row map must outlive the copy that reads it
    VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
    s->n = nk;
    s->utt = utt;
    return VB_OK;
}

extern "C" int vb_vae_stream_active(vb_vae_stream s, int32_t *utterances) {
    if (!s) return -1;
    if (utterances)
        for (int r = 0; r < s->n; r++) utterances[r] = s->utt[r];
    return s->n;
}

extern "C" void vb_vae_stream_destroy(vb_ctx *ctx, vb_vae_stream s) {
    if (!s) return;
    if (ctx) cudaStreamSynchronize(ctx->stream);
    for (void *p : s->allocs) cudaFree(p);
    if (s->work) cudaFree(s->work);
    delete s;
}

extern "C" int vb_vae_stream_conv_cache_count(vb_vae_stream s) { return s ? 20 : 0; }
extern "C" int vb_vae_stream_upconv_cache_count(vb_vae_stream s) { return s ? 6 : 0; }
extern "C" int vb_vae_stream_patch_samples(vb_vae_stream s) {
    return s ? s->patch_size * vae_upsample(s->vae->cfg) : 0;
}
extern "C" size_t vb_vae_stream_state_bytes(vb_vae_stream s) { return s ? s->state_bytes : 0; }

extern "C" int vb_vae_stream_decode(vb_ctx *ctx, vb_vae_stream s, const float *latent, int n_timesteps,
                                    float *audio) {
    if (!ctx || !s || !latent || !audio || n_timesteps <= 0) return VB_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(latent) | reinterpret_cast<uintptr_t>(audio)) % 16)
        return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_stream_decode: latent and audio must be 16-byte aligned");
    const vb_vae v = s->vae;
    const vb_vae_config &c = v->cfg;
    const int n = s->n, L = c.latent_dim, D = c.decoder_dim;
    // largest activation of one level, per buffer
    size_t need = (size_t)n * n_timesteps * std::max(L, D);
    {
        size_t T = (size_t)n_timesteps;
        for (int b = 0; b < 6; b++) {
            T *= c.rates[b];
            need = std::max(need, (size_t)n * T * (D >> (b + 1)));
        }
        if (T * (size_t)n > 0x7fffffffULL) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_stream_decode: too long");
    }
    if (need > s->work_floats) {
        if (s->work) {
            VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
            cudaFree(s->work);
            s->work = nullptr;
            s->work_floats = 0;
        }
        void *p = nullptr;
        if (cudaMalloc(&p, need * 9 * sizeof(float)) != cudaSuccess)
            return set_error(ctx, VB_ERR_OOM, "vb_vae_stream_decode: %zu bytes of activations", need * 36);
        s->work = static_cast<float *>(p);
        s->work_floats = need;
    }
    float *X0 = s->work, *XA = X0 + need, *XB = XA + need, *TB = XB + need, *H = TB + need;
    float *AH = H + need, *AL = AH + 2 * need;     // tf32 hi/lo operand (a transposed conv reads 2 x its input)
    const int p = s->parity, q = p ^ 1;
    int rc;
    // One conv as a GEMM: on the tensor cores when `tw` holds its tf32
    // weights (the operand is then already split into AH/AL), else SIMT.
    auto gemm = [&](const VaeGemm &g, Tf32Weight &tw) -> int {
        if (!tw.hi) return launch_vae_gemm(ctx, g);
        GemmEpi e;
        e.y = g.out_h;
        e.bias = g.bias;
        e.cb = g.Cb;
        e.skip = g.skip;
        e.out_x = g.out_x;
        e.alpha = g.alpha;
        e.sr_scale = g.sr_scale;
        e.sr_bias = g.sr_bias;
        return launch_gemm_tf32(ctx, tw, AH, AL, g.M, e);
    };
    // model.0: depthwise k7 over the latent (no Snake before model.1)
    const bool t_in = v->in_pw_t.hi != nullptr;
    rc = launch_dw7(ctx, latent, s->cache_in[p], s->cache_in[q], v->in_dw_w, v->in_dw_b, nullptr, t_in ? AH : X0,
                    t_in ? AL : nullptr, n, n_timesteps, L, 1);
    if (rc) return rc;
    // model.1: pointwise L -> D; emits block 0's input: snake(alpha)(sr(h))
    {
        VaeGemm g{};
        g.A = X0; g.Ka = L; g.B = v->in_pw_w; g.M = n * n_timesteps; g.N = D; g.K = L;
        g.bias = v->in_pw_b; g.Cb = D; g.out_x = XA;
        g.alpha = v->blk[0].alpha; g.sr_scale = v->blk[0].sr_scale; g.sr_bias = v->blk[0].sr_bias;
        if ((rc = gemm(g, v->in_pw_t))) return rc;
    }
    int T = n_timesteps;
    for (int b = 0; b < 6; b++) {
        VaeBlock &B = v->blk[b];
        // transposed conv: rows [x(q-1) | x(q)] -> s output times of Co
        {
            if (B.up_t.hi) {
                const int64_t items = (int64_t)n * T * 2 * (B.ci / 4);
                vae_split_prev_kernel<<<(unsigned)((items + 255) / 256), 256, 0, ctx->stream>>>(
                    XA, s->cache_up[b], AH, AL, (int64_t)n * T, T, B.ci);
                VB_LAUNCH_CHECK(ctx, "vae_split_prev");
            }
            VaeGemm g{};
            g.A = XA; g.Ka = B.ci; g.prev = s->cache_up[b]; g.T_in = T;
            g.B = B.up_w; g.M = n * T; g.N = B.s * B.co; g.K = 2 * B.ci;
            g.bias = B.up_b; g.Cb = B.co; g.out_h = H; g.out_x = XB; g.alpha = B.res[0].alpha0;
            if ((rc = gemm(g, B.up_t))) return rc;
        }
        // its history: the last (Snake-activated) input row of every stream
        VB_CHECK(ctx, cudaMemcpy2DAsync(s->cache_up[b], sizeof(float) * B.ci, XA + (size_t)(T - 1) * B.ci,
                                        sizeof(float) * T * B.ci, sizeof(float) * B.ci, n, cudaMemcpyDeviceToDevice,
                                        ctx->stream));
        T *= B.s;
        for (int u = 0; u < 3; u++) {
            VaeResUnit &R = B.res[u];
            const bool tr = R.pw_t.hi != nullptr;
            rc = launch_dw7(ctx, XB, s->cache_res[b][u][p], s->cache_res[b][u][q], R.dw_w, R.dw_b, R.alpha2,
                            tr ? AH : TB, tr ? AL : nullptr, n, T, B.co, VAE_DIL[u]);
            if (rc) return rc;
            VaeGemm g{};
            g.A = TB; g.Ka = B.co; g.B = R.pw_w; g.M = n * T; g.N = B.co; g.K = B.co;
            g.bias = R.pw_b; g.Cb = B.co; g.skip = H;
            if (u < 2) {            // skip of the next unit, and its Snake input
                g.out_h = H; g.out_x = XB; g.alpha = B.res[u + 1].alpha0;
            } else if (b < 5) {     // next block's sr_cond + Snake input
                g.out_x = XA; g.alpha = v->blk[b + 1].alpha;
                g.sr_scale = v->blk[b + 1].sr_scale; g.sr_bias = v->blk[b + 1].sr_bias;
            } else {                // model.8 Snake before the output conv
                g.out_x = XA; g.alpha = v->out_alpha;
            }
            if ((rc = gemm(g, R.pw_t))) return rc;
        }
    }
    // model.9 + tanh
    {
        const int C = D >> 6;
        const size_t smem = sizeof(float) * ((size_t)(OUT7_T + 6) * (C + 1) + (size_t)C * 7);
        if (smem > 48 * 1024) return set_error(ctx, VB_ERR_INVALID_ARG, "vb_vae_stream_decode: output conv too wide");
        dim3 grid((unsigned)((T + OUT7_T - 1) / OUT7_T), (unsigned)n);
        vae_out7_kernel<<<grid, OUT7_T, smem, ctx->stream>>>(XA, s->cache_out[p], s->cache_out[q], v->out_w, v->out_b,
                                                             audio, T, C);
        VB_LAUNCH_CHECK(ctx, "vae_out7");
    }
    s->parity = q;
    return VB_OK;
}
