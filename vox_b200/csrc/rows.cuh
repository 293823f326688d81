// Interface between the row operators' public entry points (norm.cu, softmax.cu) and their TMA row pipeline
// (rows.cu).
#pragma once

#include "common.cuh"

namespace voxcuda {

enum NormKind { kRms = 0, kLn = 1, kLnMod = 2, kAdaLn = 3, kAdaLnGated = 4 };

struct NormArgs {
    const void *x;
    const float *w;      // RMS / LN weight (f32) or NULL
    const float *b;      // LN bias (f32) or NULL
    const void *shift;   // adaLN [B][D] (dtype)
    const void *scale;   // adaLN [B][D] (dtype)
    const void *gate;    // adaLN [B][D] (dtype) or NULL
    const void *res;     // adaLN residual [rows][n] (dtype) or NULL
    void *y;
    int64_t rows, n;
    int64_t T;           // rows per batch (adaLN)
    FastDiv tdiv;        // division by T for row indices below 2^32 (set by the launcher)
    float eps;
    float inv_n;         // 1 / n
};

// Residual update + RMSNorm: h += d (* ls), xn = w * (h * inv) (kernels.cpp:822-825, 833).
struct AddRmsArgs {
    void *h;             // [rows][n] (dtype), updated in place
    const void *d;       // [rows][n] (dtype)
    const float *ls;     // per-channel layer scale [n] or NULL
    const float *w;      // RMSNorm weight [n]
    void *xn;            // [rows][n] (dtype)
    int64_t rows, n;
    float eps;
};

// Status returned by the pipeline launchers when the shape or alignment does not fit the pipeline (the caller then
// takes its general path).
constexpr int kPipeNotApplicable = 1;

// TMA row pipeline for the norm kinds; VOX_CUDA_OK, a negative status, or kPipeNotApplicable.
int launch_norm_pipe(int kind, int dtype, const NormArgs &a, cudaStream_t st, const char *name);
// TMA row pipeline for the residual update + RMSNorm; VOX_CUDA_OK, a negative status, or kPipeNotApplicable.
int launch_add_rms_pipe(int dtype, const AddRmsArgs &a, cudaStream_t st);
// TMA row pipeline for the row reductions (same fixed order as the direct kernel in reduce.cu); VOX_CUDA_OK, a
// negative status, or kPipeNotApplicable.
int launch_reduce_pipe(const void *x, float *out, int64_t rows, int64_t n, int op, int dtype, cudaStream_t st);
// TMA row pipeline for the causal softmax; VOX_CUDA_OK, a negative status, or kPipeNotApplicable.
int launch_softmax_pipe(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len, int64_t pos0,
                        cudaStream_t st);

// Reads and clears the quantized GEMV's device error flag into *flags (gemv.cu); VOX_CUDA_OK or VOX_CUDA_ERR_DEVICE.
int gemv_take_device_error(unsigned int *flags);
// The same for the F5 step's attention kernel (f5.cu).
int f5_take_device_error(unsigned int *flags);

}  // namespace voxcuda
