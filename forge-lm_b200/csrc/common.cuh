// common.cuh — shared device helpers for libforge_b200 (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define FB2_DEV __device__ __forceinline__

namespace fb2 {

constexpr int kWarp = 32;

// TF32 halves of an fp32 value for the 3xTF32 tensor-core products:
// x = hi + lo with hi = x rounded to TF32 and lo = (x - hi) rounded to TF32.
// Round to the nearest TF32 value (ties to even), kept in an fp32 container.
FB2_DEV float tf32_round(float x) {
    const uint32_t b = __float_as_uint(x);
    if ((b & 0x7F800000u) == 0x7F800000u) return x;  // inf / nan unchanged
    return __uint_as_float((b + 0x0FFFu + ((b >> 13) & 1u)) & 0xFFFFE000u);
}
FB2_DEV void tf32_split(float x, float& hi, float& lo) {
    hi = tf32_round(x);
    lo = tf32_round(x - hi);
}
// The same rounding in one instruction (cvt.rn: to nearest, ties to even;
// the 13 low bits cleared explicitly).
FB2_DEV float tf32_rn(float x) {
    uint32_t r;
    asm("cvt.rn.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r & 0xFFFFE000u);
}
FB2_DEV void tf32_split_rn(float x, float& hi, float& lo) {
    hi = tf32_rn(x);
    lo = tf32_rn(x - hi);
}

constexpr float kLnEps = 1e-5f;  // LayerNorm eps (src/LLM.Core/Model/Layers.cs:106)

FB2_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
FB2_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// tanh-approximation GELU with the reference constants
// (src/LLM.Core/Tensor/CpuBackend.cs:25-26, 510-514).
FB2_DEV float gelu_tanh(float v) {
    // MathF.Sqrt(2f / MathF.PI) evaluated in float is 0x3f4c4229 (one ulp below
    // the float nearest sqrt(2/pi), which the ILGPU kernel uses).
    const float c = __uint_as_float(0x3f4c4229u);
    const float coeff = 0.044715f;
    float u = c * (v + coeff * v * v * v);
    return 0.5f * v * (1.0f + tanhf(u));
}

// Order-preserving map float -> uint32 (larger float -> larger key).  NaN maps
// to 0, the smallest key, the position Array.Sort<float> gives NaN.
FB2_DEV uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0u;  // NaN
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
FB2_DEV float key_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// Loads that must observe data written earlier in the same kernel by other
// CTAs: bypass L1 (which is not coherent across SMs).
FB2_DEV float ld_cg(const float* p) { return __ldcg(p); }
FB2_DEV float4 ld_cg4(const float4* p) { return __ldcg(p); }

// Streaming read-only weight load: do not keep in L1.
// Programmatic dependent launch: the kernels of a decode step are launched
// with programmatic stream serialization, so a kernel's launch and prologue
// overlap its predecessor; every kernel waits here for the predecessor grid
// to complete before touching global memory (a no-op without the attribute).
FB2_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

FB2_DEV uint2 ld_stream_u2(const uint2* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
FB2_DEV float4 ld_stream4(const float4* p);
// Weight element types of the HBM-bound decode kernels: WF32 reads fp32
// weights, WBF16 reads bf16 weights (4 per 8-byte load) and widens them
// exactly to fp32.  load4(base, i) = elements 4i .. 4i+3.
struct WF32 {
    using T = float;
    static FB2_DEV float4 load4(const T* base, size_t i) { return ld_stream4(reinterpret_cast<const float4*>(base) + i); }
};
struct WBF16 {
    using T = unsigned short;  // bf16 bits
    static FB2_DEV float4 load4(const T* base, size_t i) {
        const uint2 u = ld_stream_u2(reinterpret_cast<const uint2*>(base) + i);
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                           __uint_as_float(u.y & 0xFFFF0000u));
    }
};

FB2_DEV float4 ld_stream4(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace fb2
