// Row normalisation entry points: RMSNorm, LayerNorm (affine and the AdaLayerNorm "modulate" form) and the fused
// adaLN block (LN -> (1+scale)*n + shift -> gate * m + residual) of the F5 DiT.
//
// Fast path (rows.cu): the TMA row pipeline, one warp per row, the row held in registers, for rows of up to
// 32*16 16-byte vectors whose start is 16-byte aligned. General path (here): one CTA per row reading the row
// from global memory once per pass, for any length and alignment. Both keep the CPU's statistics (f32 sum of squares
// for RMSNorm, f64 mean and variance for LayerNorm/adaLN) and its rounding order.
#include "rows.cuh"

namespace voxcuda {
namespace {

constexpr int kRowThreads = 256;

// Output of one element for every kind, in the CPU's rounding order.
template <int KIND>
__device__ __forceinline__ float norm_out(float x, float meanf, float inv, float w, float b, float sc, float sh, float g,
                                          float r) {
    if (KIND == kRms) return __fmul_rn(w, __fmul_rn(x, inv));                             // kernels.cpp:711
    const float nrm = __fmul_rn(__fsub_rn(x, meanf), inv);
    if (KIND == kLn) return __fadd_rn(__fmul_rn(nrm, w), b);                              // kernels.cpp:722
    if (KIND == kLnMod) return __fadd_rn(__fmul_rn(__fadd_rn(1.0f, w), nrm), b);          // nn.cpp:262
    const float m = __fadd_rn(__fmul_rn(nrm, __fadd_rn(1.0f, sc)), sh);                   // f5.cpp:630
    if (KIND == kAdaLn) return m;
    return __fadd_rn(r, __fmul_rn(g, m));                                                 // f5.cpp:674
}

// ------------------------------------------------------------------ general path: one CTA per row

__device__ __forceinline__ double block_sum_d(double v, double *sh) {
    v = warp_sum_d(v);
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[wid] = v;
    __syncthreads();
    double t = lane < int(blockDim.x >> 5) ? sh[lane] : 0.0;
    return warp_sum_d(t);
}
__device__ __forceinline__ float block_sum_f(float v, float *sh) {
    v = warp_sum(v);
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[wid] = v;
    __syncthreads();
    float t = lane < int(blockDim.x >> 5) ? sh[lane] : 0.f;
    return warp_sum(t);
}

template <int DT, int KIND>
__global__ void __launch_bounds__(kRowThreads) norm_row_kernel(NormArgs a) {
    pdl_enter();
    using V = Vec<DT>;
    __shared__ double shd[32];
    __shared__ float shf[32];
    for (int64_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const int64_t base = r * a.n;
        float meanf = 0.f, inv;
        if (KIND == kRms) {
            float ss = 0.f;
            for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) {
                const float v = V::load1(a.x, base + i);
                ss = __fadd_rn(ss, __fmul_rn(v, v));
            }
            ss = block_sum_f(ss, shf);
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(a.n)), a.eps)));
        } else {
            double s = 0.0;
            for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) s += double(V::load1(a.x, base + i));
            const double mean = block_sum_d(s, shd) / double(a.n);
            double v = 0.0;
            for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) {
                const double d = double(V::load1(a.x, base + i)) - mean;
                v = __dadd_rn(v, __dmul_rn(d, d));
            }
            const double var = block_sum_d(v, shd) / double(a.n);
            meanf = float(mean);
            inv = float(1.0 / sqrt(var + double(a.eps)));
        }
        __syncthreads();  // every thread has read x before any thread of this row writes y (y may equal x)
        const int64_t batch = (KIND >= kAdaLn) ? r / a.T : 0;
        for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) {
            const float f = V::load1(a.x, base + i);
            float o;
            if (KIND == kLn && !a.w) {
                const float nrm = __fmul_rn(__fsub_rn(f, meanf), inv);
                o = a.b ? __fadd_rn(nrm, a.b[i]) : nrm;
            } else {
                const float wv = (KIND <= kLnMod && a.w) ? a.w[i] : 1.0f;
                const float bv = (KIND <= kLnMod && a.b) ? a.b[i] : 0.0f;
                float sc = 0.f, sh = 0.f, g = 0.f, rv = 0.f;
                if (KIND >= kAdaLn) {
                    sc = V::load1(a.scale, batch * a.n + i);
                    sh = V::load1(a.shift, batch * a.n + i);
                }
                if (KIND == kAdaLnGated) {
                    g = V::load1(a.gate, batch * a.n + i);
                    rv = V::load1(a.res, base + i);
                }
                o = norm_out<KIND>(f, meanf, inv, wv, bv, sc, sh, g, rv);
            }
            V::store1(a.y, base + i, o);
        }
        __syncthreads();
    }
}

// Residual update + RMSNorm, one CTA per row (any length / alignment): pass 1 sums the squares of h + d * ls,
// pass 2 recomputes h + d * ls (so bf16 rows normalise the f32 sum, as the row pipeline does) and writes it to h
// and w * (h * inv) to xn. Each thread writes only the elements it reads.
template <int DT>
__global__ void __launch_bounds__(kRowThreads) add_rms_row_kernel(AddRmsArgs a) {
    pdl_enter();
    using V = Vec<DT>;
    __shared__ float shf[32];
    for (int64_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const int64_t base = r * a.n;
        float ss = 0.f;
        for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) {
            const float d = V::load1(a.d, base + i);
            const float hn = __fadd_rn(V::load1(a.h, base + i), a.ls ? __fmul_rn(d, a.ls[i]) : d);  // kernels.cpp:822-825
            ss = fmaf(hn, hn, ss);
        }
        ss = block_sum_f(ss, shf);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(a.n)), a.eps)));
        for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) {
            const float d = V::load1(a.d, base + i);
            const float hn = __fadd_rn(V::load1(a.h, base + i), a.ls ? __fmul_rn(d, a.ls[i]) : d);
            V::store1(a.h, base + i, hn);
            V::store1(a.xn, base + i, __fmul_rn(a.w[i], __fmul_rn(hn, inv)));  // kernels.cpp:711
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ dispatch

template <int DT, int KIND>
int launch_norm(const NormArgs &a, cudaStream_t st, const char *name) {
    const int rc = launch_norm_pipe(KIND, DT, a, st, name);
    if (rc != kPipeNotApplicable) return rc;
    const int64_t cap = int64_t(sm_count()) * 8;
    const int g = int(a.rows < cap ? a.rows : cap);
    launch_k(norm_row_kernel<DT, KIND>, g, kRowThreads, 0, st, a);
    return check_launch(name);
}

template <int KIND>
int dispatch_norm(int dtype, const NormArgs &a, void *stream, const char *name) {
    if (a.rows == 0) return VOX_CUDA_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == VOX_CUDA_F32) return launch_norm<VOX_CUDA_F32, KIND>(a, st, name);
    return launch_norm<VOX_CUDA_BF16, KIND>(a, st, name);
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_rmsnorm(const void *x, const float *w, void *y, int64_t rows, int64_t n, float eps, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_rmsnorm: dtype must be F32 or BF16");
    VOX_REQUIRE(rows >= 0 && n > 0, "vox_cuda_rmsnorm: bad shape");
    VOX_REQUIRE(rows == 0 || (x && w && y), "vox_cuda_rmsnorm: NULL pointer");
    NormArgs a{x, w, nullptr, nullptr, nullptr, nullptr, nullptr, y, rows, n, 1, FastDiv(1u), eps, 1.0f / float(n)};
    return dispatch_norm<kRms>(dtype, a, stream, "vox_cuda_rmsnorm");
}

int vox_cuda_layernorm(const void *x, const float *w, const float *b, void *y, int64_t rows, int64_t n, float eps, int modulate,
                       int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_layernorm: dtype must be F32 or BF16");
    VOX_REQUIRE(rows >= 0 && n > 0, "vox_cuda_layernorm: bad shape");
    VOX_REQUIRE(rows == 0 || (x && y), "vox_cuda_layernorm: NULL pointer");
    VOX_REQUIRE(!modulate || (w && b), "vox_cuda_layernorm: modulate needs w and b");
    NormArgs a{x, w, b, nullptr, nullptr, nullptr, nullptr, y, rows, n, 1, FastDiv(1u), eps, 1.0f / float(n)};
    if (modulate) return dispatch_norm<kLnMod>(dtype, a, stream, "vox_cuda_layernorm");
    return dispatch_norm<kLn>(dtype, a, stream, "vox_cuda_layernorm");
}

int vox_cuda_adaln(const void *x, const void *shift, const void *scale, const void *gate, const void *residual, void *y, int64_t B,
                   int64_t T, int64_t D, float eps, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_adaln: dtype must be F32 or BF16");
    VOX_REQUIRE(B >= 0 && T >= 0 && D > 0, "vox_cuda_adaln: bad shape");
    VOX_REQUIRE((gate == nullptr) == (residual == nullptr), "vox_cuda_adaln: gate and residual go together");
    if (B * T == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(x && shift && scale && y, "vox_cuda_adaln: NULL pointer");
    NormArgs a{x, nullptr, nullptr, shift, scale, gate, residual, y, B * T, D, T, FastDiv(1u), eps, 1.0f / float(D)};
    if (gate) return dispatch_norm<kAdaLnGated>(dtype, a, stream, "vox_cuda_adaln");
    return dispatch_norm<kAdaLn>(dtype, a, stream, "vox_cuda_adaln");
}

int vox_cuda_add_rmsnorm(void *h, const void *delta, const float *layer_scale, const float *w, void *xn, int64_t rows, int64_t n,
                         float eps, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_add_rmsnorm: dtype must be F32 or BF16");
    VOX_REQUIRE(rows >= 0 && n > 0, "vox_cuda_add_rmsnorm: bad shape");
    if (rows == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(h && delta && w && xn, "vox_cuda_add_rmsnorm: NULL pointer");
    const AddRmsArgs a{h, delta, layer_scale, w, xn, rows, n, eps};
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int rc = launch_add_rms_pipe(dtype, a, st);
    if (rc != kPipeNotApplicable) return rc;
    const int64_t cap = int64_t(sm_count()) * 8;
    const int g = int(rows < cap ? rows : cap);
    if (dtype == VOX_CUDA_F32) launch_k(add_rms_row_kernel<VOX_CUDA_F32>, g, kRowThreads, 0, st, a);
    else launch_k(add_rms_row_kernel<VOX_CUDA_BF16>, g, kRowThreads, 0, st, a);
    return check_launch("vox_cuda_add_rmsnorm");
}

}  // extern "C"
