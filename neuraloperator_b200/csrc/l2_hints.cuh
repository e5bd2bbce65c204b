// L2 eviction-priority hints for the spectral block's kernels (PTX createpolicy + .L2::cache_hint).
//
// One forward streams x (read once) and y (written once) through L2 while the kept spectra it passes
// between kernels are small (C2: 69 MB each way, L2 126 MB).  The producing kernel stores a spectrum with
// evict_last and the consuming kernel reads it with evict_first, activations and weights move with
// evict_first, so the spectra can be read back from L2 instead of HBM.  Hints change no result and no
// device setting.
#pragma once

#include <stdint.h>

namespace nop {
namespace l2 {

__device__ __forceinline__ uint64_t evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ float ld(const float* a, uint64_t pol) {
    float v;
    asm volatile("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(a), "l"(pol));
    return v;
}

__device__ __forceinline__ float2 ld2(const void* a, uint64_t pol) {
    float2 v;
    asm volatile("ld.global.nc.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;" : "=f"(v.x), "=f"(v.y) : "l"(a), "l"(pol));
    return v;
}

__device__ __forceinline__ float4 ld4(const void* a, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(a), "l"(pol));
    return v;
}

__device__ __forceinline__ void st(float* a, float v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(a), "f"(v), "l"(pol) : "memory");
}

__device__ __forceinline__ void st2(void* a, const float2& v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(a), "f"(v.x), "f"(v.y), "l"(pol)
                 : "memory");
}

__device__ __forceinline__ void st4(void* a, const float4& v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(a), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w), "l"(pol)
                 : "memory");
}

// 32-byte store (one sector)
__device__ __forceinline__ void st8(void* a, const float4& x, const float4& y, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8}, %9;" ::"l"(a), "f"(x.x),
                 "f"(x.y), "f"(x.z), "f"(x.w), "f"(y.x), "f"(y.y), "f"(y.z), "f"(y.w), "l"(pol)
                 : "memory");
}

// 16-byte async copy, zero-filled when !valid (src-size 0), with an L2 policy
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid, uint64_t pol) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;\n" ::"r"(sa), "l"(gmem),
                 "r"(valid ? 16 : 0), "l"(pol)
                 : "memory");
}

}  // namespace l2
}  // namespace nop
