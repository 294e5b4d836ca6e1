// vb_quant.cu -- weight upload/repack and Q8_0 (de)quantization kernels.
//
// GGUF Q8_0 stores each 32-weight block as {fp16 d; int8 qs[32]} = 34 bytes,
// contiguous along K.  That stride defeats 16-byte vector loads, so the
// weight is repacked once at registration: qs become a row-major int8
// [N][K] matrix (every 16-byte chunk aligned) and the scales a separate fp16
// [N][K/32] matrix.  The reference dequantizes the same blocks on the host
// (src/model_loader.c:317-331); these kernels do it on the device.
#include "vb_common.cuh"
#include "vb_kernels.cuh"
#include "vb_device.cuh"

namespace vb {

// One thread per block: split a GGUF chunk of `rows` rows into qs/scales.
__global__ void repack_q8_0_kernel(const uint8_t *__restrict__ raw, int64_t rows, int64_t nb,
                                   int8_t *__restrict__ qs, uint16_t *__restrict__ sc) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    const uint8_t *blk = raw + i * Q8_BYTES;
    const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);   // 34*i is even
    sc[i] = h[0];
    uint32_t words[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        uint32_t lo = h[1 + 2 * j], hi = h[2 + 2 * j];
        words[j] = lo | (hi << 16);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(qs + i * QK);
    dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
    dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
}

int weight_upload(vb_ctx *ctx, int type, int64_t K, int64_t N, const void *host, size_t nbytes, vb_weight *out) {
    if (type != VB_TYPE_Q8_0 && type != VB_TYPE_F16 && type != VB_TYPE_F32)
        return set_error(ctx, VB_ERR_INVALID_ARG, "weight type %d not supported (F32=0, F16=1, Q8_0=8)", type);
    if (type == VB_TYPE_Q8_0 && K % QK)
        return set_error(ctx, VB_ERR_INVALID_ARG, "Q8_0 weight K=%lld is not a multiple of 32", (long long)K);
    size_t want = type == VB_TYPE_Q8_0 ? (size_t)(N * (K / QK)) * Q8_BYTES
                                       : (size_t)(N * K) * (type == VB_TYPE_F16 ? 2u : 4u);
    if (nbytes != want)
        return set_error(ctx, VB_ERR_INVALID_ARG, "weight bytes %zu != expected %zu", nbytes, want);
    if (fault_injected("alloc")) return set_error(ctx, VB_ERR_OOM, "weight: injected allocation fault");
    VB_CHECK(ctx, cudaSetDevice(ctx->device));
    vb_weight w = new vb_weight_s();
    w->type = type;
    w->K = K;
    w->N = N;
    if (type != VB_TYPE_Q8_0) {
        if (cudaMalloc(&w->data, want) != cudaSuccess) {
            delete w;
            return set_error(ctx, VB_ERR_OOM, "weight allocation of %zu bytes failed", want);
        }
        w->device_bytes = want;
        cudaError_t e = cudaMemcpyAsync(w->data, host, want, cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            weight_free(ctx, w);
            return check_cuda(ctx, e, "weight upload");
        }
        *out = w;
        return VB_OK;
    }
    const int64_t nb = K / QK;
    size_t qs_bytes = (size_t)(N * K), sc_bytes = (size_t)(N * nb) * 2u;
    if (cudaMalloc(&w->data, qs_bytes) != cudaSuccess || cudaMalloc((void **)&w->scales, sc_bytes) != cudaSuccess) {
        weight_free(ctx, w);
        return set_error(ctx, VB_ERR_OOM, "Q8_0 weight allocation failed");
    }
    w->device_bytes = qs_bytes + sc_bytes;
    // stage the GGUF bytes in chunks of <= 64 MiB and repack on the device
    const size_t row_bytes = (size_t)nb * Q8_BYTES;
    int64_t rows_per = (int64_t)((64u << 20) / row_bytes);
    if (rows_per < 1) rows_per = 1;
    if (rows_per > N) rows_per = N;
    void *stage = nullptr;
    cudaError_t e = cudaMalloc(&stage, (size_t)rows_per * row_bytes);
    for (int64_t r0 = 0; e == cudaSuccess && r0 < N; r0 += rows_per) {
        int64_t rows = (N - r0 < rows_per) ? N - r0 : rows_per;
        e = cudaMemcpyAsync(stage, (const uint8_t *)host + (size_t)r0 * row_bytes, (size_t)rows * row_bytes,
                            cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) break;
        int64_t nthr = rows * nb;
        repack_q8_0_kernel<<<(unsigned)((nthr + 255) / 256), 256, 0, ctx->stream>>>(
            (const uint8_t *)stage, rows, nb, (int8_t *)w->data + r0 * K, w->scales + r0 * nb);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    }
    if (stage) cudaFree(stage);
    if (e != cudaSuccess) {
        weight_free(ctx, w);
        return check_cuda(ctx, e, "Q8_0 weight upload/repack");
    }
    *out = w;
    return VB_OK;
}

void weight_free(vb_ctx *ctx, vb_weight w) {
    if (!w) return;
    if (ctx) cudaStreamSynchronize(ctx->stream);
    if (w->data) cudaFree(w->data);
    if (w->scales) cudaFree(w->scales);
    delete w;
}

// dst[o][j] = value of flat element j*out_dim + o of a registered weight, as
// exact F32: the stop predictor reads its two weights in [in][out] storage
// order (W_buf[j*hs + i], H_buf[2*j + o], src/gen_stop.c:126-135,180-195)
// after dequantizing them with read_tensor_f32 (:28-74).  Flat element f of
// a registered [N][K] weight is row f / K, column f % K.
__global__ void transpose_f32_kernel(const void *__restrict__ data, const uint16_t *__restrict__ sc, int type,
                                     int64_t K, int64_t in_dim, int64_t out_dim, float *__restrict__ dst) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= in_dim * out_dim) return;
    const int64_t o = i / in_dim, j = i % in_dim;
    const int64_t f = j * out_dim + o, n = f / K, k = f % K;
    float v;
    if (type == VB_TYPE_Q8_0)
        v = __fmul_rn((float)static_cast<const int8_t *>(data)[n * K + k], h2f(sc[n * (K / QK) + k / QK]));
    else if (type == VB_TYPE_F16)
        v = h2f(static_cast<const uint16_t *>(data)[n * K + k]);
    else
        v = static_cast<const float *>(data)[n * K + k];
    dst[i] = v;
}

int weight_transpose_f32(vb_ctx *ctx, vb_weight src, int64_t in_dim, int64_t out_dim, vb_weight *out) {
    *out = nullptr;
    if (!src || in_dim <= 0 || out_dim <= 0 || src->K * src->N != in_dim * out_dim)
        return set_error(ctx, VB_ERR_INVALID_ARG, "weight re-layout: %lld x %lld values expected", (long long)in_dim,
                         (long long)out_dim);
    if (fault_injected("alloc")) return set_error(ctx, VB_ERR_OOM, "weight: injected allocation fault");
    vb_weight w = new vb_weight_s();
    w->type = VB_TYPE_F32;
    w->K = in_dim;
    w->N = out_dim;
    w->device_bytes = (size_t)(in_dim * out_dim) * 4u;
    if (cudaMalloc(&w->data, w->device_bytes) != cudaSuccess) {
        delete w;
        return set_error(ctx, VB_ERR_OOM, "weight re-layout: allocation of %zu bytes failed", (size_t)(in_dim * out_dim) * 4u);
    }
    const int64_t n = in_dim * out_dim;
    transpose_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(src->data, src->scales, src->type, src->K,
                                                                             in_dim, out_dim, (float *)w->data);
    const int rc = check_launch(ctx, "transpose_f32");
    if (rc) {
        weight_free(ctx, w);
        return rc;
    }
    *out = w;
    return VB_OK;
}

// One warp per 32-value block; output in the GGUF 34-byte layout.
__global__ void quantize_q8_0_kernel(const float *__restrict__ x, int64_t nblocks, uint8_t *__restrict__ out,
                                     int rule) {
    int64_t blk = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (blk >= nblocks) return;
    float v = x[blk * QK + lane];
    int q;
    uint16_t dh;
    q8_quant_warp(v, rule, q, dh);
    uint8_t *b = out + blk * Q8_BYTES;
    b[2 + lane] = (uint8_t)(int8_t)q;
    if (lane == 0) *reinterpret_cast<uint16_t *>(b) = dh;
}

int launch_quantize_q8_0(vb_ctx *ctx, const float *x, int64_t K, int64_t M, void *blocks, int rule) {
    if (K % QK) return set_error(ctx, VB_ERR_INVALID_ARG, "quantize: K=%lld not a multiple of 32", (long long)K);
    int64_t nblocks = M * (K / QK);
    if (nblocks == 0) return VB_OK;
    quantize_q8_0_kernel<<<(unsigned)((nblocks + 7) / 8), 256, 0, ctx->stream>>>(x, nblocks, (uint8_t *)blocks,
                                                                                   rule);
    VB_LAUNCH_CHECK(ctx, "quantize_q8_0");
    return VB_OK;
}

// w = (float)qs[j] * fp16->fp32(d): one exact fp32 product per value.
__global__ void dequantize_q8_0_kernel(const uint8_t *__restrict__ blocks, int64_t n, float *__restrict__ y) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t *b = blocks + (i / QK) * Q8_BYTES;
    float d = h2f(*reinterpret_cast<const uint16_t *>(b));
    y[i] = __fmul_rn((float)(int8_t)b[2 + (i % QK)], d);
}

int launch_dequantize_q8_0(vb_ctx *ctx, const void *blocks, int64_t n, float *y) {
    if (n % QK) return set_error(ctx, VB_ERR_INVALID_ARG, "dequantize: n=%lld not a multiple of 32", (long long)n);
    if (n == 0) return VB_OK;
    dequantize_q8_0_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>((const uint8_t *)blocks, n, y);
    VB_LAUNCH_CHECK(ctx, "dequantize_q8_0");
    return VB_OK;
}

// Embedding lookup (gen_forward_text, src/gen_prompt.c:67-131): row i of y
// is table row ids[i] as F32; an id outside [0, N) reads row 0, as the
// reference clamps it.  Q8_0 rows are (float)qs * fp16->fp32(d), one exact
// product per value; F16 rows are the exact widening; F32 rows are copied.
// One CTA per output row, 8 values per thread per pass.
template <int TYPE>
__global__ void get_rows_kernel(const void *__restrict__ data, const uint16_t *__restrict__ scales, int64_t K,
                                int64_t N, const int32_t *__restrict__ ids, float *__restrict__ y) {
    const int64_t i = blockIdx.x;
    int64_t id = ids[i];
    if (id < 0 || id >= N) id = 0;
    float *yr = y + i * K;
    for (int64_t k = (int64_t)threadIdx.x * 8; k < K; k += (int64_t)blockDim.x * 8) {
        float v[8];
        if (TYPE == VB_TYPE_Q8_0) {
            const int2 q = __ldg(reinterpret_cast<const int2 *>(static_cast<const int8_t *>(data) + id * K + k));
            const float d = h2f(__ldg(scales + id * (K / QK) + k / QK));
            const int8_t *qb = reinterpret_cast<const int8_t *>(&q);
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = __fmul_rn((float)qb[e], d);
        } else if (TYPE == VB_TYPE_F16) {
            const int4 h = __ldg(reinterpret_cast<const int4 *>(static_cast<const uint16_t *>(data) + id * K + k));
            const uint16_t *hb = reinterpret_cast<const uint16_t *>(&h);
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = h2f(hb[e]);
        } else {
            const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(data) + id * K + k);
            const float4 a = __ldg(src), b = __ldg(src + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
        reinterpret_cast<float4 *>(yr + k)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(yr + k)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

int launch_get_rows(vb_ctx *ctx, vb_weight w, const int32_t *ids, int64_t n, float *y) {
    if (w->K % 8)
        return set_error(ctx, VB_ERR_INVALID_ARG, "get_rows: row width K=%lld is not a multiple of 8", (long long)w->K);
    if (reinterpret_cast<uintptr_t>(y) % 16)
        return set_error(ctx, VB_ERR_INVALID_ARG, "get_rows: output is not 16-byte aligned");
    if (n > 0x7fffffffLL) return set_error(ctx, VB_ERR_INVALID_ARG, "get_rows: too many rows");
    if (n == 0) return VB_OK;
    const int threads = (int)std::min<int64_t>(256, (w->K / 8 + 31) / 32 * 32);
    switch (w->type) {
        case VB_TYPE_Q8_0:
            get_rows_kernel<VB_TYPE_Q8_0><<<(unsigned)n, threads, 0, ctx->stream>>>(w->data, w->scales, w->K, w->N, ids, y);
            break;
        case VB_TYPE_F16:
            get_rows_kernel<VB_TYPE_F16><<<(unsigned)n, threads, 0, ctx->stream>>>(w->data, nullptr, w->K, w->N, ids, y);
            break;
        default:
            get_rows_kernel<VB_TYPE_F32><<<(unsigned)n, threads, 0, ctx->stream>>>(w->data, nullptr, w->K, w->N, ids, y);
            break;
    }
    VB_LAUNCH_CHECK(ctx, "get_rows");
    return VB_OK;
}

}  // namespace vb
