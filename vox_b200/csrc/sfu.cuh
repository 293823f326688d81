// Special-function-unit approximations used where the full-range CUDA functions cost more instructions than an
// HBM-bound kernel can afford. Errors: ex2.approx.ftz.f32 and rcp.approx.ftz.f32 are within a few ulp of the exact
// results (the PTX ISA's documented bounds); denormal inputs flush to zero.
#pragma once

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

}  // namespace voxcuda
