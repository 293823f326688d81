// Special-function-unit approximations used where the full-range CUDA functions cost more instructions than an
// HBM-bound kernel can afford. Errors: ex2.approx.ftz.f32 and rcp.approx.ftz.f32 are within a few ulp of the exact
// results (the PTX ISA's documented bounds); denormal inputs flush to zero.
#pragma once

#include "common.cuh"

namespace voxcuda {

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU, tanh form (f5.cpp:93-96): 0.5 x (1 + tanh(k (x + 0.044715 x^3))), tanh(z) = 1 - 2 / (1 + e^(2z)) with the SFU's
// ex2 and rcp (absolute error ~1e-7); two elements per call.
__device__ __forceinline__ float2 gelu_tanh_f2(float2 x) {
    const float2 z = mul2(bc2(0.7978845608028654f), fma2(mul2(bc2(0.044715f), x), mul2(x, x), x));
    const float2 e = mul2(bc2(2.8853900817779268f), z);  // e^(2z) = 2^(2z log2(e))
    const float2 d = add2(bc2(1.0f), make_float2(ex2_approx(e.x), ex2_approx(e.y)));
    const float2 th = fma2(bc2(-2.0f), make_float2(rcp_approx(d.x), rcp_approx(d.y)), bc2(1.0f));
    return mul2(mul2(bc2(0.5f), x), add2(bc2(1.0f), th));
}

// GELU, erf form (kernels.hpp:106, nn.cpp:87-96): x * Phi(x), Phi from the normal tail of Abramowitz & Stegun 26.2.17,
// two elements per call.
__device__ __forceinline__ float2 gelu_erf_f2(float2 x) {
    const float2 a = make_float2(fabsf(x.x), fabsf(x.y));
    const float2 d = fma2(bc2(0.2316419f), a, bc2(1.0f));
    const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
    // b_k / sqrt(2 pi) of A&S 26.2.17
    float2 p = fma2(bc2(0.530702714f), t, bc2(-0.726576013f));  // 1.330274429, -1.821255978 (/ sqrt(2 pi))
    p = fma2(p, t, bc2(0.710706871f));                            // 1.781477937
    p = fma2(p, t, bc2(-0.142248368f));                           // -0.356563782
    p = fma2(p, t, bc2(0.127414796f));                            // 0.319381530
    p = mul2(p, t);
    const float2 g = mul2(mul2(a, a), bc2(-0.72134752f));         // exp(-a^2 / 2) = 2^(-a^2 log2(e) / 2)
    const float2 xq = mul2(x, mul2(make_float2(ex2_approx(g.x), ex2_approx(g.y)), p));  // x * Q(|x|)
    const float2 hi = fma2(xq, bc2(-1.0f), x);                    // x - x Q(|x|)
    return make_float2(x.x >= 0.f ? hi.x : xq.x, x.y >= 0.f ? hi.y : xq.y);
}

}  // namespace voxcuda
