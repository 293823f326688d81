// Scaled, causally truncated row softmax (f32): y = softmax(scale * x) over each row's visible prefix, zeros after.
//
// Vox never materialises the causal mask: kernels.cpp:812-819 truncates query i's row to its n = pos0+i+1 visible
// keys, scales the dot products, runs softmax_inplace (kernels.cpp:725-732: max, exp(x - max), float sum,
// multiply by 1/sum) and leaves nothing beyond. Here the visible prefix is the only part of x that is read
// (rounded up to a 16-byte vector); the full row of y is written, zeros past the prefix, which equals the
// "-inf above the diagonal" form since exp(-inf - max) = 0.
//
// Fast path (rows.cu): the TMA row pipeline, one warp per row, the visible prefix staged by bulk copy and held in
// registers (n <= 2048). General path (here): one CTA per row, three passes over global memory.
#include <math.h>

#include "rows.cuh"

namespace voxcuda {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ int64_t visible_len(int64_t r, int64_t n, int64_t q_len, int64_t pos0) {
    if (q_len <= 0) return n;
    const int64_t v = (r % q_len) + pos0 + 1;
    return v < n ? (v > 0 ? v : 0) : n;
}

__device__ __forceinline__ float block_reduce(float v, float *sh, bool is_max) {
    v = is_max ? warp_max(v) : warp_sum(v);
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[wid] = v;
    __syncthreads();
    float t = lane < int(blockDim.x >> 5) ? sh[lane] : (is_max ? -INFINITY : 0.f);
    return is_max ? warp_max(t) : warp_sum(t);
}

__global__ void __launch_bounds__(kRowThreads)
    softmax_row_kernel(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len, int64_t pos0) {
    pdl_enter();
    __shared__ float sh[32];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int64_t vis = visible_len(r, n, q_len, pos0);
        const float *xr = x + r * n;
        float *yr = y + r * n;
        float mx = -INFINITY;
        for (int64_t i = threadIdx.x; i < vis; i += blockDim.x) mx = fmaxf(mx, __fmul_rn(scale, xr[i]));
        mx = block_reduce(mx, sh, true);
        float sum = 0.f;
        for (int64_t i = threadIdx.x; i < vis; i += blockDim.x) sum = __fadd_rn(sum, expf(__fsub_rn(__fmul_rn(scale, xr[i]), mx)));
        sum = block_reduce(sum, sh, false);
        const float inv = __fdiv_rn(1.0f, sum);
        __syncthreads();  // all reads of x done before y (which may equal x) is written
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
            yr[i] = i < vis ? __fmul_rn(expf(__fsub_rn(__fmul_rn(scale, xr[i]), mx)), inv) : 0.f;
        __syncthreads();
    }
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" int vox_cuda_softmax_rows(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len, int64_t pos0,
                                     void *stream) {
    VOX_REQUIRE(rows >= 0 && n > 0 && q_len >= 0 && pos0 >= 0, "vox_cuda_softmax_rows: bad shape");
    if (rows == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(x && y, "vox_cuda_softmax_rows: NULL pointer");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int rc = launch_softmax_pipe(x, y, rows, n, scale, q_len, pos0, st);
    if (rc != kPipeNotApplicable) return rc;
    const int64_t cap = int64_t(sm_count()) * 8;
    const int g = int(rows < cap ? rows : cap);
    launch_k(softmax_row_kernel, g, kRowThreads, 0, st, x, y, rows, n, scale, q_len, pos0);
    return check_launch("vox_cuda_softmax_rows");
}
