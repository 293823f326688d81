// The cross-GPU step of the deterministic global sum, in the library: NCCL communicators and one call that runs a
// shard's slot partials, the all-reduce of the 840 f64 slots and the fixed-order fold (vox_cuda_global_sum).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2: the copy a host process such as PyTorch already loaded, else the
// system's), so the library keeps no link-time dependency on it and single-GPU users never load it. Communicators are
// created non-blocking (ncclConfig_t.blocking = 0): every NCCL call returns at once, and the library polls
// ncclCommGetAsyncError against a deadline; a communicator that misses its deadline (a peer that never joins, a
// collective that never completes) is aborted (ncclCommAbort, which also ends its kernels) and the call returns
// VOX_CUDA_ERR_DEVICE, so a rank learns of a lost peer on the host instead of hanging. The all-reduce adds the slot
// vectors element-wise; every shard owns whole slots and writes zeros elsewhere, so the sum is exact and the result
// identical for 1..8 GPUs. No counterpart in the reference (Vox runs one device per process).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

struct vox_cuda_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0;
    bool aborted = false;
};

namespace voxcuda {
namespace {

struct Nccl {
    void *h = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*init_all)(ncclComm_t *, int, const int *) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const Nccl &nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        for (const char *name : {"libnccl.so.2", "libnccl.so"}) {
            n.h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
            if (n.h) break;
        }
        if (!n.h) return;
        auto sym = [](const char *s) { return dlsym(n.h, s); };
        n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(sym("ncclGetUniqueId"));
        n.init_rank_config = reinterpret_cast<decltype(n.init_rank_config)>(sym("ncclCommInitRankConfig"));
        n.init_all = reinterpret_cast<decltype(n.init_all)>(sym("ncclCommInitAll"));
        n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(sym("ncclAllReduce"));
        n.async_error = reinterpret_cast<decltype(n.async_error)>(sym("ncclCommGetAsyncError"));
        n.abort = reinterpret_cast<decltype(n.abort)>(sym("ncclCommAbort"));
        n.destroy = reinterpret_cast<decltype(n.destroy)>(sym("ncclCommDestroy"));
        n.group_start = reinterpret_cast<decltype(n.group_start)>(sym("ncclGroupStart"));
        n.group_end = reinterpret_cast<decltype(n.group_end)>(sym("ncclGroupEnd"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(sym("ncclGetErrorString"));
        n.ok = n.get_unique_id && n.init_rank_config && n.init_all && n.all_reduce && n.async_error && n.abort && n.destroy &&
               n.group_start && n.group_end && n.error_string;
    });
    return n;
}

int nccl_missing(const char *what) { return set_error(VOX_CUDA_ERR_UNSUPPORTED, std::string(what) + ": libnccl.so.2 not found (NCCL >= 2.14)"); }

std::string nccl_msg(ncclResult_t r) {
    const Nccl &n = nccl();
    return n.error_string ? n.error_string(r) : ("NCCL error " + std::to_string(int(r)));
}

constexpr int kDefaultDeadlineMs = 30000;

int abort_comm(vox_cuda_comm *c, const std::string &msg) {
    nccl().abort(c->comm);
    c->aborted = true;
    return set_error(VOX_CUDA_ERR_DEVICE, msg + " (communicator aborted)");
}

// Between polls: yield for the first 2 ms (a non-blocking enqueue usually completes within microseconds, and a 50 us
// sleep there left the GPU idle behind every small all-reduce), then sleep 50 us.
void poll_pause(std::chrono::steady_clock::time_point t0) {
    if (std::chrono::steady_clock::now() - t0 < std::chrono::milliseconds(2)) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
}

// Polls the communicator until its pending call has completed (ncclSuccess), failed, or the deadline passed (then the
// communicator is aborted). VOX_CUDA_OK or VOX_CUDA_ERR_DEVICE.
int settle(vox_cuda_comm *c, int timeout_ms, const char *what) {
    const Nccl &n = nccl();
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = n.async_error(c->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return VOX_CUDA_OK;
        if (st != ncclInProgress) return abort_comm(c, std::string(what) + ": " + nccl_msg(st));
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
            return abort_comm(c, std::string(what) + ": deadline of " + std::to_string(timeout_ms) + " ms passed (a peer did not join)");
        poll_pause(t0);
    }
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_comm_unique_id(void *id) {
    VOX_REQUIRE(id != nullptr, "vox_cuda_comm_unique_id: id is NULL");
    const Nccl &n = nccl();
    if (!n.ok) return nccl_missing("vox_cuda_comm_unique_id");
    ncclUniqueId u;
    const ncclResult_t r = n.get_unique_id(&u);
    if (r != ncclSuccess) return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_comm_unique_id: " + nccl_msg(r));
    static_assert(sizeof(ncclUniqueId) == VOX_CUDA_COMM_ID_BYTES, "unique id size");
    std::memcpy(id, &u, sizeof(u));
    return VOX_CUDA_OK;
}

int vox_cuda_comm_init_rank(const void *id, int nranks, int rank, int timeout_ms, vox_cuda_comm **out) {
    VOX_REQUIRE(id && out && nranks >= 1 && rank >= 0 && rank < nranks, "vox_cuda_comm_init_rank: bad arguments");
    *out = nullptr;
    const Nccl &n = nccl();
    if (!n.ok) return nccl_missing("vox_cuda_comm_init_rank");
    auto *c = new vox_cuda_comm();
    c->nranks = nranks, c->rank = rank;
    cudaGetDevice(&c->device);
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = n.init_rank_config(&c->comm, nranks, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_comm_init_rank: " + nccl_msg(r));
    }
    const int rc = settle(c, timeout_ms > 0 ? timeout_ms : kDefaultDeadlineMs, "vox_cuda_comm_init_rank");
    if (rc != VOX_CUDA_OK) {
        delete c;
        return rc;
    }
    *out = c;
    return VOX_CUDA_OK;
}

int vox_cuda_comm_init_all(int ndev, const int *devices, vox_cuda_comm **comms) {
    VOX_REQUIRE(ndev >= 1 && devices && comms, "vox_cuda_comm_init_all: bad arguments");
    const Nccl &n = nccl();
    if (!n.ok) return nccl_missing("vox_cuda_comm_init_all");
    std::vector<ncclComm_t> cs(size_t(ndev), nullptr);
    const ncclResult_t r = n.init_all(cs.data(), ndev, devices);
    if (r != ncclSuccess) return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_comm_init_all: " + nccl_msg(r));
    for (int i = 0; i < ndev; ++i) {
        comms[i] = new vox_cuda_comm();
        comms[i]->comm = cs[size_t(i)], comms[i]->nranks = ndev, comms[i]->rank = i, comms[i]->device = devices[i];
    }
    return VOX_CUDA_OK;
}

int vox_cuda_comm_group_start(void) {
    const Nccl &n = nccl();
    if (!n.ok) return nccl_missing("vox_cuda_comm_group_start");
    const ncclResult_t r = n.group_start();
    return r == ncclSuccess ? VOX_CUDA_OK : set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_comm_group_start: " + nccl_msg(r));
}

int vox_cuda_comm_group_end(void) {
    const Nccl &n = nccl();
    if (!n.ok) return nccl_missing("vox_cuda_comm_group_end");
    const ncclResult_t r = n.group_end();
    return r == ncclSuccess || r == ncclInProgress ? VOX_CUDA_OK : set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_comm_group_end: " + nccl_msg(r));
}

int vox_cuda_comm_wait(vox_cuda_comm *c, void *stream, int timeout_ms) {
    VOX_REQUIRE(c != nullptr, "vox_cuda_comm_wait: comm is NULL");
    if (c->aborted) return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_comm_wait: the communicator was aborted");
    const Nccl &n = nccl();
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int lim = timeout_ms > 0 ? timeout_ms : kDefaultDeadlineMs;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return VOX_CUDA_OK;
        if (q != cudaErrorNotReady) return check_launch("vox_cuda_comm_wait");
        ncclResult_t as = ncclSuccess;
        n.async_error(c->comm, &as);
        if (as != ncclSuccess && as != ncclInProgress) return abort_comm(c, "vox_cuda_comm_wait: " + nccl_msg(as));
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(lim))
            return abort_comm(c, "vox_cuda_comm_wait: deadline of " + std::to_string(lim) + " ms passed before the stream's work completed");
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

void vox_cuda_comm_destroy(vox_cuda_comm *c) {
    if (!c) return;
    const Nccl &n = nccl();
    if (n.ok && c->comm && !c->aborted) n.destroy(c->comm);  // an aborted communicator is already released
    delete c;
}

int vox_cuda_global_sum(const void *x, int64_t rows, int64_t n, int64_t row0, int64_t total_rows, float *rowsum_scratch, double *slots,
                        double *out, int dtype, vox_cuda_comm *comm, void *stream) {
    VOX_REQUIRE(out != nullptr, "vox_cuda_global_sum: out is NULL");
    VOX_REQUIRE(comm == nullptr || !comm->aborted, "vox_cuda_global_sum: the communicator was aborted");
    int rc = vox_cuda_global_sum_partials(x, rows, n, row0, total_rows, rowsum_scratch, slots, dtype, stream);
    if (rc != VOX_CUDA_OK) return rc;
    if (comm && comm->nranks > 1) {
        const Nccl &nc = nccl();
        if (!nc.ok) return nccl_missing("vox_cuda_global_sum");
        const ncclResult_t r = nc.all_reduce(slots, slots, VOX_CUDA_GLOBAL_SUM_SLOTS, ncclFloat64, ncclSum, comm->comm,
                                             reinterpret_cast<cudaStream_t>(stream));
        if (r != ncclSuccess && r != ncclInProgress) return set_error(VOX_CUDA_ERR_DEVICE, "vox_cuda_global_sum: all-reduce: " + nccl_msg(r));
        if (r == ncclInProgress && (rc = settle(comm, kDefaultDeadlineMs, "vox_cuda_global_sum")) != VOX_CUDA_OK) return rc;
    }
    return vox_cuda_global_sum_finish(slots, out, stream);
}

}  // extern "C"
