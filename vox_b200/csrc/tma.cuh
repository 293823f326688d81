// TMA row staging: 1-D bulk copies (cp.async.bulk, global -> shared) completed on mbarriers, and the per-warp row
// pipeline that the row operators (RMSNorm, LayerNorm, adaLN, causal softmax) run on.
//
// Each warp owns STAGES shared-memory buffers and their mbarriers. Lane 0 issues the bulk copies of the warp's
// next rows STAGES rows ahead; the warp waits for a row's barrier, moves the row into registers, hands the buffer
// back to lane 0 for the row STAGES ahead, and computes. Row data in flight costs no registers, so every warp
// keeps loads in flight while it computes, which is what a row operator needs to run at HBM speed.
//
// Each copy lands in the shared memory of the issuing CTA only (a plain shared::cluster destination of a CTA that is
// a cluster of one); no copy is broadcast to other CTAs.
// Every wait is bounded: a wait that gives up records VOX_CUDA_DEVERR_TIMEOUT in a device flag, waits (bounded
// again) for every copy of the warp still in flight (the one it gave up on included), and the warp stops;
// vox_cuda_device_error() reads and clears the flag.
#pragma once

#include "common.cuh"

namespace voxcuda {

// Device-side error flag of the pipelines (a bit set by a kernel that gave up a wait). The library is built without
// relocatable device code, so every translation unit that includes this header has its own flag; each of them
// exposes it through take_device_error() and vox_cuda_device_error() gathers them all.
static __device__ unsigned int g_device_error = 0;
constexpr unsigned int kDevErrTimeout = 1u;
// A wait gives up after this much time on the GPU's global timer (ns), read every 32 polls (each try_wait may also
// suspend the warp for a hardware-chosen time). The limit is a device variable of the translation unit so that a test
// can shorten it (vox_cuda_test_row_stall); every kernel reads it only once its first poll has failed.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
static __device__ uint64_t g_wait_limit_ns = kWaitLimitNs;
// Test hook of the row pipelines: the row whose stage barrier is told to expect 16 bytes more than its copies
// deliver (every copy still lands, the phase never completes, the wait runs out); -1 = none.
static __device__ int64_t g_stall_row = -1;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// One arrival on `bar` (release: this thread's earlier writes are visible to the thread whose wait completes).
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait of a whole warp for the phase of `parity` to complete. Every lane polls (so every lane acquires the
// phase) and every decision is warp-uniform (the time limit too); false, with the device error flag set, if the phase
// has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = *(volatile uint64_t *)&g_wait_limit_ns;
    for (uint32_t i = 1;; ++i) {
        if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
        if ((i & 31u) == 0 && __any_sync(0xffffffffu, globaltimer_ns() - t0 > limit)) break;
    }
    if ((threadIdx.x & 31) == 0) atomicOr(&g_device_error, kDevErrTimeout);
    return false;
}
// Raises the transaction count the current phase of `bar` waits for, without an arrival.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Orders this thread's earlier generic-proxy accesses of shared memory before later async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) from global memory into this CTA's shared
// memory, completing `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

constexpr int kPipeWarps = 4;  // warps per CTA of a row pipeline

// Shared memory of a row pipeline CTA: kPipeWarps * STAGES mbarriers, then kPipeWarps * STAGES buffers.
__host__ __device__ constexpr uint32_t pipe_bar_bytes(int stages) { return ((kPipeWarps * stages * 8 + 127) / 128) * 128; }
__host__ __device__ constexpr uint32_t pipe_smem_bytes(int stages, uint32_t stage_bytes) {
    return pipe_bar_bytes(stages) + uint32_t(kPipeWarps * stages) * stage_bytes;
}

// The per-warp row pipeline. Op provides kMinBlocks (the CTAs per SM its register budget is sized for) and
//   __device__ uint32_t issue(int64_t r, uint8_t *buf, uint64_t *bar) const   // lane 0: expect_tx + bulk copies
//   template <class Next> __device__ void run(int64_t r, const uint8_t *buf, int lane, Next next) const
// run() reads the row from buf into registers, calls next() (which releases buf for the row STAGES ahead), then
// computes and stores the row.
template <class Op, int STAGES>
__global__ void __launch_bounds__(kPipeWarps * 32, Op::kMinBlocks) row_pipe_kernel(Op op, int64_t rows, uint32_t stage_bytes) {
    pdl_enter();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * STAGES;
    uint8_t *bufs = smem + pipe_bar_bytes(STAGES) + size_t(warp) * STAGES * stage_bytes;
    const int64_t gw = int64_t(blockIdx.x) * kPipeWarps + warp;
    const int64_t nw = int64_t(gridDim.x) * kPipeWarps;
    if (gw >= rows) return;
    const int64_t stall = lane == 0 ? g_stall_row : -1;  // test hook (-1 in normal use)
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        mbar_init_fence();
#pragma unroll
        for (int s = 0; s < STAGES; ++s) {
            const int64_t r = gw + s * nw;
            if (r == stall) mbar_expect_tx(&bars[s], 16);
            if (r < rows) op.issue(r, bufs + s * stage_bytes, &bars[s]);
        }
    }
    uint32_t pending = 0;  // bit s: a copy into stage s is in flight (warp-uniform)
#pragma unroll
    for (int t = 0; t < STAGES; ++t)
        if (gw + t * nw < rows) pending |= 1u << t;
    __syncwarp();
    uint32_t parity = 0;  // bit s: parity of the next phase of stage s
    int s = 0;
    for (int64_t r = gw; r < rows; r += nw) {
        if (!mbar_wait_warp(&bars[s], (parity >> s) & 1u)) {
            // give up: let every copy of the warp still in flight land (bounded), the one waited for included,
            // before the CTA's shared memory can be reused
            for (int t = 0; t < STAGES; ++t)
                if ((pending >> t) & 1u) mbar_wait_warp(&bars[t], (parity >> t) & 1u);
            return;
        }
        parity ^= 1u << s;
        pending &= ~(1u << s);
        uint8_t *buf = bufs + s * stage_bytes;
        uint64_t *bar = &bars[s];
        const int64_t r_next = r + int64_t(STAGES) * nw;
        const int cur = s;
        op.run(r, buf, lane, [&]() {
            __syncwarp();
            if (r_next < rows) {
                if (lane == 0) {
                    fence_proxy_async();
                    if (r_next == stall) mbar_expect_tx(bar, 16);
                    op.issue(r_next, buf, bar);
                }
                pending |= 1u << cur;
            }
        });
        s = (s + 1 == STAGES) ? 0 : s + 1;
    }
}

// Launches row_pipe_kernel<Op, STAGES> over `rows` rows: a balanced persistent grid of at most one resident wave.
template <class Op, int STAGES>
int launch_row_pipe(const Op &op, int64_t rows, uint32_t stage_bytes, cudaStream_t st, const char *name) {
    const uint32_t smem = pipe_smem_bytes(STAGES, stage_bytes);
    if (int(smem) > smem_optin()) return set_error(VOX_CUDA_ERR_UNSUPPORTED, std::string(name) + ": row too long for shared memory");
    auto kern = row_pipe_kernel<Op, STAGES>;
    if (smem > 48 * 1024) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
            return check_launch(name);
    }
    const int g = balanced_grid(rows, kPipeWarps, resident_blocks((const void *)kern, kPipeWarps * 32, smem));
    launch_k(kern, g, kPipeWarps * 32, smem, st, op, rows, stage_bytes);
    return check_launch(name);
}

// The flag read and cleared in one atomic step on the device (a flag raised by a kernel still running on another
// stream is either taken now or left set for the next read, never lost).
static __device__ unsigned int g_device_error_taken = 0;
static __global__ void take_device_error_kernel() { g_device_error_taken = atomicExch(&g_device_error, 0u); }

// Reads and clears this translation unit's device error flag (host side; the legacy default stream, so it follows
// the work of every blocking stream). VOX_CUDA_OK or VOX_CUDA_ERR_DEVICE.
static inline int take_device_error(unsigned int *flags) {
    unsigned int v = 0;
    take_device_error_kernel<<<1, 1>>>();
    if (cudaGetLastError() != cudaSuccess || cudaMemcpyFromSymbol(&v, g_device_error_taken, sizeof(v)) != cudaSuccess)
        return VOX_CUDA_ERR_DEVICE;
    *flags |= v;
    return VOX_CUDA_OK;
}

// Test hook (host side): sets this translation unit's wait limit (ns; 0 restores the default) and stalled row.
static inline int set_wait_test_hook(int64_t stall_row, uint64_t limit_ns) {
    const uint64_t lim = limit_ns ? limit_ns : kWaitLimitNs;
    if (cudaMemcpyToSymbol(g_stall_row, &stall_row, sizeof(stall_row)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_wait_limit_ns, &lim, sizeof(lim)) != cudaSuccess)
        return VOX_CUDA_ERR_DEVICE;
    return VOX_CUDA_OK;
}

}  // namespace voxcuda
