// vb_common.cuh -- shared definitions of the B200 hot-path library.
//
// One vb_ctx = one device + one stream, used by one host thread at a time
// (the reference runtime is single-device and non-reentrant,
// src/ggml_backend.c:244-246).  Every entry point returns a vcpm_status code
// and never aborts; the message of the last failure is kept per context.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>
#include <string>
#include <vector>
#include <mutex>

#include "vcpm_b200.h"

namespace vb {

constexpr int QK = 32;          // Q8_0 block length
constexpr int Q8_BYTES = 34;    // GGUF Q8_0 block: fp16 d + 32 int8

// ---------------------------------------------------------------- errors
struct Status {
    int code = VB_OK;
    std::string msg;
};

// Host-side fault injection: VB_FAULT=alloc|launch makes the matching step
// fail before the device is touched (failure paths are testable without a
// GPU fault).
bool fault_injected(const char *what);

// --------------------------------------------------------------- workspace
// A growable device arena owned by the context.  Grows only outside of
// stream capture; kernels address scratch through it.
struct Arena {
    void *ptr = nullptr;
    size_t bytes = 0;
};

struct RopeTable {
    int head_dim = 0;
    float theta = 0.f;
    int use_factors = 0;
    int max_pos = 0;
    float *d_cs = nullptr;   // [max_pos][head_dim] (cos, sin) pairs
};

}  // namespace vb

// A registered weight, repacked for 16-byte coalesced loads:
//   Q8_0: qs int8 [N][K] + scales fp16 [N][K/32] (split from the 34-byte
//         GGUF blocks), F16: fp16 [N][K], F32: fp32 [N][K].
struct vb_weight_s {
    int type = 0;
    int64_t K = 0, N = 0;
    void *data = nullptr;
    uint16_t *scales = nullptr;
    size_t device_bytes = 0;
    alignas(64) unsigned char tmap[128];   // tensor-core path: TMA descriptor of the weight tiles
    bool tmap_ok = false;
    alignas(64) unsigned char tmap_i8[128];   // int8 tensor-core path (Q8_0): 128 x 128 swizzled tiles
    bool tmap_i8_ok = false;
};

// Host F32->BF16->F32 (round to nearest even, quiet NaN).
float vb_host_bf16(float x);

struct vb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;          // stream all work is enqueued on
    cudaStream_t own_stream_handle = nullptr;
    bool own_stream = false;
    int qrule = VB_QRULE_X86;
    std::string last_error;
    vb::Arena ws;                       // general scratch
    vb::Arena attn_ws;                  // attention chunk partials
    std::vector<vb::RopeTable> ropes;   // cached rotary tables
    int sm_count = 0;
    size_t smem_optin = 0;
    bool use_gemm = true;               // tensor-core path for M >= 16 (VB_GEMM=0 disables)
    int gemm_i8 = 1;                    // Q8_0 on the int8 tensor cores: 1 where faster (the default),
                                        // 2 always (VB_GEMM_I8=2), 0 never (VB_GEMM_I8=0: the fp16 split form)
    void *gemm = nullptr;               // tensor-core path state (vb_gemm.cu)
    void *attn_noalloc = nullptr;       // device address of vb_attention_noalloc's fixed scratch on this device
    long long dep_wait_limit = 0;       // streaming kernel: cycles of a wait on other CTAs (0 = default)
};

namespace vb {

int set_error(vb_ctx *ctx, int code, const char *fmt, ...);
int check_cuda(vb_ctx *ctx, cudaError_t e, const char *what);
int check_launch(vb_ctx *ctx, const char *what);
int arena_reserve(vb_ctx *ctx, Arena &a, size_t bytes);
inline int ws_reserve(vb_ctx *ctx, size_t bytes) { return arena_reserve(ctx, ctx->ws, bytes); }
const RopeTable *rope_table(vb_ctx *ctx, int head_dim, float theta, int use_factors, int need_pos);
// The (cos, sin) table of positions 0..max_pos-1 on the host.
void rope_table_host(int head_dim, float theta, int use_factors, int max_pos, std::vector<float> &cs);
const float *longrope_short_factors();

// ------------------------------------------------------- device helpers
// F32 -> BF16 -> F32 with round-to-nearest-even and quiet NaN: the same
// integer formula the oracle uses, so results are bit-identical.
__device__ __forceinline__ float bf16r(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(((u >> 16) | 0x40u) << 16);
    u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
    return __uint_as_float(u);
}

__device__ __forceinline__ uint16_t bf16_bits(float x) {
    return (uint16_t)(__float_as_uint(bf16r(x)) >> 16);
}

__device__ __forceinline__ float bf16_to_f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint16_t f2h(float x) { return __half_as_ushort(__float2half_rn(x)); }

// silu(x) = x / (1 + expf(-x)) with IEEE division (CUDA expf).
__device__ __forceinline__ float silu_f(float x) {
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace vb

#define VB_CHECK(ctx, expr)                                    \
    do {                                                       \
        cudaError_t _e = (expr);                               \
        if (_e != cudaSuccess) return vb::check_cuda((ctx), _e, #expr); \
    } while (0)

#define VB_LAUNCH_CHECK(ctx, what)                             \
    do {                                                       \
        int _rc = vb::check_launch((ctx), (what));             \
        if (_rc) return _rc;                                   \
    } while (0)
