// Row reductions (sum / max / L2 norm) and the two device steps of the deterministic cross-shard global sum.
//
// Rows of up to 16 KB run on the TMA row pipeline (rows.cu); longer or unaligned rows on the direct kernel here.
// Both follow one reduction order (fixed, so results are bitwise reproducible and restatable on the CPU): the row is cut
// into "vectors" of W elements (4 for f32, 8 for bf16; the last one may be short); lane l of the row's warp takes
// vectors l, l+32, l+64, ... in order and adds element k of each vector into accumulator k % 4; the lane's value
// is (acc0 + acc1) + (acc2 + acc3); the 32 lane values are folded by an xor butterfly over offsets 16, 8, 4, 2, 1.
// Every add and multiply is rounded separately (no FMA). The aligned vector path and the scalar path follow the
// same order. max uses fmaxf; L2 = sqrt(sum of x*x).
//
// Global sum (no counterpart in Vox, which has no multi-device code): the global tensor's rows are split into
// VOX_CUDA_GLOBAL_SUM_SLOTS = 840 = lcm(1..8) slots, slot s = rows [floor(s*R/840), floor((s+1)*R/840)). A slot's
// partial is the f64 sum of its rows' f32 row sums: lane l of the slot's warp adds rows l, l+32, ... in order, then
// the xor butterfly. A shard owning whole slots writes its partials and zeros elsewhere; the element-wise sum of
// all shards' slot vectors (one NCCL all-reduce) is exact, and the finish step folds the 840 slots in a fixed
// order. The result therefore does not depend on the number of shards.
#include "rows.cuh"

namespace voxcuda {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kUnroll = 8;

template <int OP>
__device__ __forceinline__ float red_step(float acc, float v) {
    if (OP == VOX_CUDA_REDUCE_MAX) return fmaxf(acc, v);
    if (OP == VOX_CUDA_REDUCE_L2) return __fadd_rn(acc, __fmul_rn(v, v));
    return __fadd_rn(acc, v);
}
template <int OP>
__device__ __forceinline__ float red_join(float a, float b) {
    return OP == VOX_CUDA_REDUCE_MAX ? fmaxf(a, b) : __fadd_rn(a, b);
}
template <int OP>
__device__ __forceinline__ float red_init() {
    return OP == VOX_CUDA_REDUCE_MAX ? -INFINITY : 0.f;
}

// One warp per row, VEC = 16-byte vector path (row start aligned, n % W == 0) or scalar path (same order).
template <int DT, int OP, bool VEC>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) row_reduce_kernel(const void *x, float *out, int64_t rows, int64_t n) {
    pdl_enter();
    using V = Vec<DT>;
    constexpr int W = V::N;
    constexpr int ES = DT == VOX_CUDA_F32 ? 4 : 2;
    const int lane = threadIdx.x & 31;
    const int64_t nvec = (n + W - 1) / W;
    const int64_t warp0 = int64_t(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
    const int64_t nwarps = int64_t(gridDim.x) * kWarpsPerBlock;
    for (int64_t r = warp0; r < rows; r += nwarps) {
        const char *xr = reinterpret_cast<const char *>(x) + r * n * ES;
        float acc[4] = {red_init<OP>(), red_init<OP>(), red_init<OP>(), red_init<OP>()};
        int64_t j = lane;
        if (VEC) {
            for (; j + 32 * (kUnroll - 1) < nvec; j += 32 * kUnroll) {
                uint4 raw[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) raw[u] = ld_stream(xr + (j + 32 * u) * 16);
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    float f[W];
                    V::unpack(raw[u], f);
#pragma unroll
                    for (int k = 0; k < W; ++k) acc[k % 4] = red_step<OP>(acc[k % 4], f[k]);
                }
            }
            for (; j < nvec; j += 32) {
                float f[W];
                V::unpack(ld_stream(xr + j * 16), f);
#pragma unroll
                for (int k = 0; k < W; ++k) acc[k % 4] = red_step<OP>(acc[k % 4], f[k]);
            }
        } else {
            for (; j < nvec; j += 32) {
                for (int k = 0; k < W; ++k) {
                    const int64_t e = j * W + k;
                    if (e < n) acc[k % 4] = red_step<OP>(acc[k % 4], V::load1(xr, e));
                }
            }
        }
        float v = red_join<OP>(red_join<OP>(acc[0], acc[1]), red_join<OP>(acc[2], acc[3]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = red_join<OP>(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) out[r] = OP == VOX_CUDA_REDUCE_L2 ? __fsqrt_rn(v) : v;
    }
}

template <int DT, int OP>
void launch_rr(const void *x, float *out, int64_t rows, int64_t n, bool vec, cudaStream_t st) {
    auto kern = vec ? row_reduce_kernel<DT, OP, true> : row_reduce_kernel<DT, OP, false>;
    const int g = balanced_grid(rows, kWarpsPerBlock, resident_blocks((const void *)kern, kWarpsPerBlock * 32, 0));
    launch_k(kern, g, kWarpsPerBlock * 32, 0, st, x, out, rows, n);
}

template <int DT>
void dispatch_rr(int op, const void *x, float *out, int64_t rows, int64_t n, bool vec, cudaStream_t st) {
    if (op == VOX_CUDA_REDUCE_SUM) launch_rr<DT, VOX_CUDA_REDUCE_SUM>(x, out, rows, n, vec, st);
    else if (op == VOX_CUDA_REDUCE_MAX) launch_rr<DT, VOX_CUDA_REDUCE_MAX>(x, out, rows, n, vec, st);
    else launch_rr<DT, VOX_CUDA_REDUCE_L2>(x, out, rows, n, vec, st);
}

int row_reduce(const void *x, float *out, int64_t rows, int64_t n, int op, int dtype, cudaStream_t st) {
    const int rc = launch_reduce_pipe(x, out, rows, n, op, dtype, st);  // rows staged by TMA (rows.cu)
    if (rc != kPipeNotApplicable) return rc;
    const int W = dtype == VOX_CUDA_F32 ? 4 : 8;
    const bool vec = n % W == 0 && aligned16(x);
    if (dtype == VOX_CUDA_F32) dispatch_rr<VOX_CUDA_F32>(op, x, out, rows, n, vec, st);
    else dispatch_rr<VOX_CUDA_BF16>(op, x, out, rows, n, vec, st);
    return check_launch("vox_cuda_row_reduce");
}

__host__ __device__ __forceinline__ int64_t slot_begin(int64_t s, int64_t R) { return (s * R) / VOX_CUDA_GLOBAL_SUM_SLOTS; }

// One warp per slot: owned slots get the fixed-order f64 sum of their row sums, the others 0.
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    slot_partials_kernel(const float *rowsum, int64_t row0, int64_t rows, int64_t R, double *slots) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int64_t s = int64_t(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
    if (s >= VOX_CUDA_GLOBAL_SUM_SLOTS) return;
    const int64_t lo = slot_begin(s, R), hi = slot_begin(s + 1, R);
    const bool owned = lo >= row0 && hi <= row0 + rows;
    double acc = 0.0;
    if (owned)
        for (int64_t r = lo + lane; r < hi; r += 32) acc += double(rowsum[r - row0]);
    acc = warp_sum_d(acc);
    if (lane == 0) slots[s] = owned ? acc : 0.0;
}

// One block of 256 threads: thread t adds slots t, t+256, ... in order; warps fold by butterfly; warp 0 folds the
// 8 warp values by butterfly.
__global__ void __launch_bounds__(256) slot_finish_kernel(const double *slots, double *out) {
    pdl_enter();
    __shared__ double sh[8];
    double acc = 0.0;
    for (int s = threadIdx.x; s < VOX_CUDA_GLOBAL_SUM_SLOTS; s += 256) acc += slots[s];
    acc = warp_sum_d(acc);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < 8 ? sh[threadIdx.x] : 0.0;
        t = warp_sum_d(t);
        if (threadIdx.x == 0) out[0] = t;
    }
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_row_reduce(const void *x, float *out, int64_t rows, int64_t n, int op, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_row_reduce: dtype must be F32 or BF16");
    VOX_REQUIRE(op == VOX_CUDA_REDUCE_SUM || op == VOX_CUDA_REDUCE_MAX || op == VOX_CUDA_REDUCE_L2, "vox_cuda_row_reduce: unknown op");
    VOX_REQUIRE(rows >= 0 && n > 0, "vox_cuda_row_reduce: bad shape");
    if (rows == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(x && out, "vox_cuda_row_reduce: NULL pointer");
    return row_reduce(x, out, rows, n, op, dtype, reinterpret_cast<cudaStream_t>(stream));
}

int vox_cuda_global_sum_partials(const void *x, int64_t rows, int64_t n, int64_t row0, int64_t total_rows, float *rowsum_scratch,
                                 double *slots, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_global_sum_partials: dtype must be F32 or BF16");
    VOX_REQUIRE(rows >= 0 && n > 0 && row0 >= 0 && total_rows >= 0 && row0 + rows <= total_rows,
                "vox_cuda_global_sum_partials: shard outside the global tensor");
    VOX_REQUIRE(slots != nullptr, "vox_cuda_global_sum_partials: slots is NULL");
    VOX_REQUIRE(rows == 0 || (x && rowsum_scratch), "vox_cuda_global_sum_partials: NULL pointer");
    // The shard must start and end on slot boundaries (slot_begin is non-decreasing in s: binary search).
    auto is_boundary = [total_rows](int64_t row) {
        int64_t lo = 0, hi = VOX_CUDA_GLOBAL_SUM_SLOTS;
        while (lo < hi) {
            const int64_t mid = (lo + hi) / 2;
            if (slot_begin(mid, total_rows) < row) lo = mid + 1;
            else hi = mid;
        }
        return slot_begin(lo, total_rows) == row;
    };
    const bool lo_ok = is_boundary(row0), hi_ok = is_boundary(row0 + rows);
    VOX_REQUIRE(lo_ok && hi_ok, "vox_cuda_global_sum_partials: shard rows are not a whole number of slots");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (rows > 0) {
        const int rc = row_reduce(x, rowsum_scratch, rows, n, VOX_CUDA_REDUCE_SUM, dtype, st);
        if (rc != VOX_CUDA_OK) return rc;
    }
    launch_k(slot_partials_kernel, (VOX_CUDA_GLOBAL_SUM_SLOTS + kWarpsPerBlock - 1) / kWarpsPerBlock, kWarpsPerBlock * 32, 0, st, 
        rowsum_scratch, row0, rows, total_rows, slots);
    return check_launch("vox_cuda_global_sum_partials");
}

int vox_cuda_global_sum_finish(const double *slots, double *out, void *stream) {
    VOX_REQUIRE(slots && out, "vox_cuda_global_sum_finish: NULL pointer");
    launch_k(slot_finish_kernel, 1, 256, 0, reinterpret_cast<cudaStream_t>(stream), slots, out);
    return check_launch("vox_cuda_global_sum_finish");
}

}  // extern "C"
