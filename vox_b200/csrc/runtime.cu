// Host plumbing of the vox_cuda C ABI: per-thread last error, device attribute cache, grid sizing, service calls.
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "common.cuh"

namespace voxcuda {

namespace {
thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
struct DevAttr {
    int sms = 0;
    int smem_optin = 0;
};
DevAttr g_attr[kMaxDevices];
std::once_flag g_attr_once[kMaxDevices];

const DevAttr &attr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        static const DevAttr fallback{148, 227 * 1024};
        return fallback;
    }
    std::call_once(g_attr_once[dev], [dev] {
        DevAttr a;
        if (cudaDeviceGetAttribute(&a.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) a.sms = 148;
        if (cudaDeviceGetAttribute(&a.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
            a.smem_optin = 48 * 1024;
        cudaGetLastError();
        g_attr[dev] = a;
    });
    return g_attr[dev];
}
}  // namespace

int set_error(int status, const std::string &msg) {
    g_last_error = msg;
    return status;
}

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return VOX_CUDA_OK;
    return set_error(VOX_CUDA_ERR_DEVICE, std::string(what) + ": " + cudaGetErrorString(e));
}

bool pdl_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("VOX_CUDA_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

int sm_count() { return attr().sms; }
int smem_optin() { return attr().smem_optin; }

int resident_blocks(const void *kernel, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<std::pair<const void *, int>, std::pair<int, size_t>>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) cudaGetLastError();
    const auto key = std::make_pair(std::make_pair(kernel, dev), std::make_pair(threads, smem));
    {
        std::lock_guard<std::mutex> g(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    const int r = per_sm * sm_count();
    std::lock_guard<std::mutex> g(mu);
    cache[key] = r;
    return r;
}

int balanced_grid(int64_t units, int64_t per_block, int resident) {
    if (units <= 0) return 1;
    const int64_t blocks_needed = (units + per_block - 1) / per_block;
    const int64_t res = resident > 0 ? resident : 1;
    const int64_t passes = (blocks_needed + res - 1) / res;
    const int64_t g = (blocks_needed + passes - 1) / passes;
    return int(g < 1 ? 1 : g);
}

int grid_for(int64_t work_items, int threads, int per_sm) {
    const int64_t need = (work_items + threads - 1) / threads;
    const int64_t cap = int64_t(sm_count()) * per_sm;
    const int64_t g = need < cap ? need : cap;
    return int(g < 1 ? 1 : g);
}

}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

const char *vox_cuda_version(void) { return "vox-cuda 0.1.0 sm_100a"; }

const char *vox_cuda_last_error(void) { return g_last_error.c_str(); }

int vox_cuda_device_count(int *count) {
    VOX_REQUIRE(count != nullptr, "vox_cuda_device_count: count is NULL");
    const cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        return set_error(VOX_CUDA_ERR_DEVICE, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
    }
    return VOX_CUDA_OK;
}

int vox_cuda_device_cc(int *cc) {
    VOX_REQUIRE(cc != nullptr, "vox_cuda_device_cc: cc is NULL");
    int dev = 0, ma = 0, mi = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&ma, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&mi, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        return set_error(VOX_CUDA_ERR_DEVICE, std::string("device query: ") + cudaGetErrorString(e));
    }
    *cc = ma * 10 + mi;
    return VOX_CUDA_OK;
}

}  // extern "C"
