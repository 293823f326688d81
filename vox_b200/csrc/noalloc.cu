// Allocation-free variant of the global sum (vox_cuda_global_sum_noalloc).
//
// Some callers cannot call cudaMalloc: code running in a real-time audio callback (cudaMalloc can block and
// synchronise the device, which breaks the callback's deadline), or plugin hosts that hand a library device buffers
// for inputs and outputs but keep every other allocation to themselves. vox_cuda_global_sum needs scratch memory for
// its row sums and its 840 slot partials; this variant keeps that scratch in one fixed array in the library's own
// device memory instead, so the caller passes only the tensor and the output.
//
// The scratch array below is a static device variable of this translation unit: it lives in the library's device
// module, so every device on which that module is loaded holds its kNoAllocScratchBytes (about 1 MB) until the
// process exits. With CUDA's lazy module loading (the default) the module, and so the array, is loaded on a device
// the first time the library needs it there, at the latest on this entry point's first call on that device. Host code
// may not use the array's name as a device address (on the host it is only a stand-in symbol); its device address is
// looked up with cudaGetSymbolAddress, with the device current, on the first call in each CUDA context, and passed to
// the kernels. That first call may load the module and block, so it is a warm-up: make it outside any real-time path
// (and before any stream capture) on every device. The address is kept together with the context it belongs to: a
// call in another context of the device (after cudaDeviceReset) looks it up again, and a failed lookup is not kept.
#include <cuda.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace voxcuda {
namespace {

// Largest tensor the entry point accepts: 262144 rows (row sums, f32) plus the 840 f64 slot partials.
constexpr int64_t kNoAllocMaxRows = 262144;
constexpr size_t kRowSumBytes = size_t(kNoAllocMaxRows) * sizeof(float);
constexpr size_t kSlotBytes = size_t(VOX_CUDA_GLOBAL_SUM_SLOTS) * sizeof(double);
constexpr size_t kNoAllocScratchBytes = kRowSumBytes + kSlotBytes;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchSlot {
    unsigned long long ctx_id = 0;  // unique id of the context the address belongs to (cuCtxGetId; never reused)
    unsigned char *addr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// The driver's cuCtxGetCurrent and cuCtxGetId, looked up once through the runtime (no link-time dependency on
// libcuda).
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);
template <class Fn>
Fn driver_fn(const char *name) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return reinterpret_cast<Fn>(p);
}

// Device address of g_noalloc_scratch in the current device's current context.
int scratch_address(unsigned char **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        return set_error(VOX_CUDA_ERR_DEVICE, std::string("vox_cuda_global_sum_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
    }
    if (dev < 0 || dev >= kMaxDevices) return set_error(VOX_CUDA_ERR_UNSUPPORTED, "vox_cuda_global_sum_noalloc: device index too large");
    static const CtxGetCurrentFn get = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
    static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
    if (!get || !get_id) return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_global_sum_noalloc: cuCtxGetCurrent / cuCtxGetId not available");
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
        // no context current on this thread yet: cudaSetDevice makes the device's primary context current (CUDA 12)
        if (cudaSetDevice(dev) != cudaSuccess || get(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
            cudaGetLastError();
            return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_global_sum_noalloc: no CUDA context on the current device");
        }
    }
    unsigned long long id = 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_global_sum_noalloc: cuCtxGetId failed");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchSlot &slot = g_scratch[dev];
    if (slot.ctx_id != id || slot.addr == nullptr) {
        void *p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (rc != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            slot = ScratchSlot{};  // not kept: the next call tries again
            return set_error(VOX_CUDA_ERR_DEVICE, std::string("vox_cuda_global_sum_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(rc));
        }
        slot.ctx_id = id;
        slot.addr = static_cast<unsigned char *>(p);
    }
    *out = slot.addr;
    return VOX_CUDA_OK;
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" int vox_cuda_global_sum_noalloc(const void *x, int64_t rows, int64_t n, double *out, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_global_sum_noalloc: dtype must be F32 or BF16");
    VOX_REQUIRE(rows >= 0 && n > 0, "vox_cuda_global_sum_noalloc: bad shape");
    VOX_REQUIRE(out != nullptr && (rows == 0 || x != nullptr), "vox_cuda_global_sum_noalloc: NULL pointer");
    VOX_REQUIRE(rows <= kNoAllocMaxRows, "vox_cuda_global_sum_noalloc: " + std::to_string(rows) +
                                             " rows exceed the limit of 262144 rows of this allocation-free variant "
                                             "(use vox_cuda_global_sum_partials with caller scratch)");
    unsigned char *scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc != VOX_CUDA_OK) return rc;
    float *rowsum = reinterpret_cast<float *>(scratch);
    double *slots = reinterpret_cast<double *>(scratch + kRowSumBytes);
    // Nothing in the scratch needs to start at zero: the partials step writes every row sum it reads and every one of
    // the 840 slots (0 for the slots it does not own) before the finish step reads them.
    const int r1 = vox_cuda_global_sum_partials(x, rows, n, 0, rows, rowsum, slots, dtype, stream);
    if (r1 != VOX_CUDA_OK) return r1;
    return vox_cuda_global_sum_finish(slots, out, stream);
}
