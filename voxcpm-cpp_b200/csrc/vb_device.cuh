// vb_device.cuh -- device-side building blocks shared by the kernels.
#pragma once

#include "vb_common.cuh"

namespace vb {

// Warp-collective Q8_0 quantization of one 32-value block, lane j holding
// value j.  d = amax/127 (IEEE division) stored as fp16 (RNE); the
// reciprocal and tie rule follow `rule` (include/vcpm_b200.h).  Every
// operation is explicitly rounded so the result is bit-identical to the CPU
// restatement of ggml's rule.
__device__ __forceinline__ void q8_quant_warp(float v, int rule, int &q, uint16_t &dh) {
    const float amax = warp_max(fabsf(v));
    const float d = __fdiv_rn(amax, 127.0f);
    dh = f2h(d);
    float id;
    if (rule == VB_QRULE_X86) id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    const float t = __fmul_rn(v, id);
    q = (rule == VB_QRULE_X86) ? __float2int_rn(t) : (int)roundf(t);
}

// 16-byte streaming load of read-once data: bypass L1 allocation and ask L2
// for a 256-byte prefetch.
__device__ __forceinline__ int4 ldg_stream(const void *p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ int dot16_i8(const int4 &a, const int4 &b) {
    int s = __dp4a(a.x, b.x, 0);
    s = __dp4a(a.y, b.y, s);
    s = __dp4a(a.z, b.z, s);
    s = __dp4a(a.w, b.w, s);
    return s;
}

// fp32 dot of 8 fp16 pairs packed in two int4 (accumulated with fma).
__device__ __forceinline__ float dot8_f16(const int4 &a, const int4 &b, float acc) {
    const __half2 *ha = reinterpret_cast<const __half2 *>(&a);
    const __half2 *hb = reinterpret_cast<const __half2 *>(&b);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 fa = __half22float2(ha[i]);
        float2 fb = __half22float2(hb[i]);
        acc = fmaf(fa.x, fb.x, acc);
        acc = fmaf(fa.y, fb.y, acc);
    }
    return acc;
}

__device__ __forceinline__ float dot4_f32(const int4 &a, const float4 &b, float acc) {
    acc = fmaf(__int_as_float(a.x), b.x, acc);
    acc = fmaf(__int_as_float(a.y), b.y, acc);
    acc = fmaf(__int_as_float(a.z), b.z, acc);
    acc = fmaf(__int_as_float(a.w), b.w, acc);
    return acc;
}

}  // namespace vb
