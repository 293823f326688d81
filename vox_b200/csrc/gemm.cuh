// Internal interface of the tcgen05 GEMM (gemm.cu): y = x . W^T (+ bias) with a fused epilogue, bf16 operands, f32
// accumulation in tensor memory. Used by the C ABI (vox_cuda_gemm_bf16) and by the F5 DiT step (f5.cu), which builds
// its GEMMs once at plan creation and replays them inside a CUDA graph.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace voxcuda {

// Epilogues of the tcgen05 GEMM (applied to the f32 accumulator of each output element).
enum GemmEpi {
    kEpiF32 = 0,          // y (f32) = acc (+ bias) (+ y if accumulate)
    kEpiBf16 = 1,         // y (bf16) = acc (+ bias)
    kEpiQkvRope = 2,      // y (bf16) = RoPE(acc + bias) on the q and k parts of a fused q|k|v projection (F5 interleaved pairs)
    kEpiGeluTanh = 3,     // y (bf16) = gelu_tanh(acc + bias)
    kEpiGeluErf = 4,      // y (bf16) = gelu_erf(acc + bias)
    kEpiGeluTanhF32 = 5,  // y (f32) = gelu_tanh(acc + bias)
    kEpiGeluErfF32 = 6,   // y (f32) = gelu_erf(acc + bias)
};

struct GemmArgs {
    int M = 0, N = 0, K = 0;          // rows of x and y, rows of W (columns of y), reduction length
    int batches = 1, groups = 1;      // z = b * groups + g: x plane z, W plane g, y offset b * y_bstride + g * y_gstride
    void *y = nullptr;
    int64_t ldy = 0;                  // row stride of y (elements)
    int64_t y_bstride = 0, y_gstride = 0;
    const float *bias = nullptr;      // [groups][N] f32, or NULL
    int accumulate = 0;               // kEpiF32: y += result
    // kEpiQkvRope: y [M][3 inner]; row r at position r % frames; heads < rope_heads of q and k rotate with cs[pos][hd/2]
    const float2 *cs = nullptr;
    int frames = 1, rope_heads = 0, hd = 64, inner = 0;
    int tile = 0;                     // 0: gemm_plan picks the tile; else 1000 * pair + BN (128, 256, 1128, 1192, ...)
    int w_early = 0;                  // 1: W is not written by the previous kernel of the stream (weights of a plan), so
                                      // its first copies may start before that kernel has ended (one-CTA tiles)
    int tma_store = 0;                // set by gemm_plan: y is written by tensor stores (GemmPlan::ty)
    int f16 = 0;                      // 1: x and W are f16, not bf16 (kEpiF32 only)
};

// A prepared GEMM: its tensor maps (x planes [z][M][K], W planes [g][N][K], bf16, 128-byte swizzle; y in 32 x 32
// boxes where its layout allows tensor stores), the tile shape and the epilogue. Built once per operand set;
// launching it allocates nothing.
struct GemmPlan {
    CUtensorMap ta, tb, ty;
    GemmArgs a;
    int bn = 128;
    bool pair = false;  // a cluster of two CTAs per 256 x 256 tile (tcgen05 cta_group::2)
    int epi = kEpiF32;
};

// Builds a plan for x (bf16, or f16 with a.f16, [batches * groups][M][K] planes, row pitch ldx elements) and W (the
// same type, [groups][N][K], row pitch ldw): K % 8 == 0, ldx and ldw multiples of 8, x and W 16-byte aligned. VOX_CUDA_OK or an error status.
int gemm_plan(const void *x, int64_t ldx, const void *w, int64_t ldw, const GemmArgs &a, int epi, GemmPlan &plan, const char *name);
// Launches a prepared GEMM on stream st.
int gemm_run(const GemmPlan &plan, cudaStream_t st, const char *name);
// Reads and clears the GEMM kernels' device error flag (bit 0: a bounded wait gave up).
int gemm_take_device_error(unsigned int *flags);

}  // namespace voxcuda
