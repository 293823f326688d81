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

}  // namespace voxcuda
