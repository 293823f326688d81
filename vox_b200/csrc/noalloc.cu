// Allocation-free variant of the global sum (vox_cuda_global_sum_noalloc).
//
// Some callers cannot call cudaMalloc: code running in a real-time audio callback (cudaMalloc can block and
// synchronise the device, which breaks the callback's deadline), or plugin hosts that hand a library device buffers
// for inputs and outputs but keep every other allocation to themselves. vox_cuda_global_sum needs scratch memory for
// its row sums and its 840 slot partials; this variant keeps that scratch in one fixed array in the library's own
// device memory instead, so the caller passes only the tensor and the output.
//
// The scratch array below is a static device variable of this translation unit: every GPU that loads the library
// holds its kNoAllocScratchBytes (about 1 MB) until the process exits. Host code may not use the array's name as a
// device address (on the host it is only a stand-in symbol); its device address is looked up once per device with
// cudaGetSymbolAddress, on that device's first call of the entry point, and passed to the kernels.
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
unsigned char *g_scratch_addr[kMaxDevices];
std::once_flag g_scratch_once[kMaxDevices];
cudaError_t g_scratch_rc[kMaxDevices];

// Device address of g_noalloc_scratch on the current device (looked up once per device, with that device current).
int scratch_address(unsigned char **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        return set_error(VOX_CUDA_ERR_DEVICE, std::string("vox_cuda_global_sum_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
    }
    if (dev < 0 || dev >= kMaxDevices) return set_error(VOX_CUDA_ERR_UNSUPPORTED, "vox_cuda_global_sum_noalloc: device index too large");
    std::call_once(g_scratch_once[dev], [dev] {
        void *p = nullptr;
        g_scratch_rc[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (g_scratch_rc[dev] != cudaSuccess) cudaGetLastError();
        g_scratch_addr[dev] = static_cast<unsigned char *>(p);
    });
    if (g_scratch_rc[dev] != cudaSuccess || g_scratch_addr[dev] == nullptr)
        return set_error(VOX_CUDA_ERR_DEVICE, std::string("vox_cuda_global_sum_noalloc: cudaGetSymbolAddress: ") +
                                                  cudaGetErrorString(g_scratch_rc[dev]));
    *out = g_scratch_addr[dev];
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
