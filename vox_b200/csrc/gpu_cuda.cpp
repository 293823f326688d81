// The C++17 host seam (include/vox_gpu_cuda.hpp) over the C ABI: bool results, failures counted and their
// messages kept in GpuCudaStats::last_error, no exception crosses the seam (src/gpu.hpp conventions).
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <string>

#include "../../include/vox_gpu_cuda.hpp"

#define VOX_CXX_API __attribute__((visibility("default")))

namespace vox {

namespace {
std::mutex g_init_mu;                 // guards device initialisation only
std::atomic<int64_t> g_ok{0}, g_failed{0};
std::mutex g_err_mu;
std::string g_last_error;
thread_local bool g_active = false;

bool done(int rc) {
    if (rc == VOX_CUDA_OK) {
        g_ok.fetch_add(1, std::memory_order_relaxed);
        return true;
    }
    g_failed.fetch_add(1, std::memory_order_relaxed);
    std::lock_guard<std::mutex> g(g_err_mu);
    g_last_error = vox_cuda_last_error();
    return false;
}
bool cuda_done(cudaError_t e, const char *what) {
    if (e == cudaSuccess) {
        g_ok.fetch_add(1, std::memory_order_relaxed);
        return true;
    }
    g_failed.fetch_add(1, std::memory_order_relaxed);
    std::lock_guard<std::mutex> g(g_err_mu);
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return false;
}
cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }
}  // namespace

VOX_CXX_API bool gpu_cuda_init(int device, std::string &err) {
    std::lock_guard<std::mutex> g(g_init_mu);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        err = "no CUDA device";
        return false;
    }
    if (device < 0 || device >= n) {
        err = "CUDA device " + std::to_string(device) + " does not exist (" + std::to_string(n) + " found)";
        return false;
    }
    cudaDeviceProp p{};
    if (cudaSetDevice(device) != cudaSuccess || cudaGetDeviceProperties(&p, device) != cudaSuccess) {
        err = std::string("cudaSetDevice: ") + cudaGetErrorString(cudaGetLastError());
        return false;
    }
    if (p.major != 10) {
        err = std::string("vox-cuda is built for sm_100a; device is ") + p.name + " (sm_" + std::to_string(p.major * 10 + p.minor) + ")";
        return false;
    }
    g_active = true;
    return true;
}

VOX_CXX_API bool gpu_cuda_active() { return g_active; }

VOX_CXX_API std::string gpu_cuda_device_name() {
    int d = 0;
    cudaDeviceProp p{};
    if (cudaGetDevice(&d) != cudaSuccess || cudaGetDeviceProperties(&p, d) != cudaSuccess) {
        cudaGetLastError();
        return "";
    }
    return p.name;
}

VOX_CXX_API GpuCudaStats gpu_cuda_stats() {
    GpuCudaStats s;
    s.calls_ok = g_ok.load();
    s.calls_failed = g_failed.load();
    std::lock_guard<std::mutex> g(g_err_mu);
    s.last_error = g_last_error;
    return s;
}

VOX_CXX_API void *gpu_cuda_alloc(size_t bytes) {
    void *p = nullptr;
    if (!cuda_done(cudaMalloc(&p, bytes), "cudaMalloc")) return nullptr;
    return p;
}
VOX_CXX_API void gpu_cuda_free(void *p) {
    if (p) cuda_done(cudaFree(p), "cudaFree");
}
VOX_CXX_API bool gpu_cuda_upload(void *dst, const void *src, size_t bytes, void *stream) {
    return cuda_done(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, S(stream)), "upload");
}
VOX_CXX_API bool gpu_cuda_download(void *dst, const void *src, size_t bytes, void *stream) {
    return cuda_done(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, S(stream)), "download");
}
VOX_CXX_API bool gpu_cuda_sync(void *stream) { return cuda_done(cudaStreamSynchronize(S(stream)), "sync"); }

VOX_CXX_API bool gpu_rmsnorm(const void *x, const float *w, int64_t rows, int64_t n, float eps, void *out, int dtype, void *stream) {
    return done(vox_cuda_rmsnorm(x, w, out, rows, n, eps, dtype, stream));
}
VOX_CXX_API bool gpu_layernorm(const void *x, const float *w, const float *b, int64_t rows, int64_t n, float eps, void *out, int dtype,
                               void *stream) {
    return done(vox_cuda_layernorm(x, w, b, out, rows, n, eps, 0, dtype, stream));
}
VOX_CXX_API bool gpu_layer_norm(void *x, int T, int C, const float *w, const float *b, float eps, bool modulate, int dtype,
                                void *stream) {
    return done(vox_cuda_layernorm(x, w, b, x, T, C, eps, modulate ? 1 : 0, dtype, stream));
}
VOX_CXX_API bool gpu_adaln(const void *x, const void *shift, const void *scale, const void *gate, const void *residual, void *out,
                           int64_t B, int64_t T, int64_t D, float eps, int dtype, void *stream) {
    return done(vox_cuda_adaln(x, shift, scale, gate, residual, out, B, T, D, eps, dtype, stream));
}
VOX_CXX_API bool gpu_softmax_causal(const float *scores, float *probs, int64_t heads, int64_t q_len, int64_t n_keys, float scale,
                                    int64_t pos0, void *stream) {
    return done(vox_cuda_softmax_rows(scores, probs, heads * q_len, n_keys, scale, q_len, pos0, stream));
}
VOX_CXX_API bool gpu_silu_mul(const void *g, const void *u, void *h, int64_t n, int dtype, void *stream) {
    return done(vox_cuda_silu_mul(g, u, h, n, dtype, stream));
}
VOX_CXX_API bool gpu_gelu(const void *x, void *y, int64_t n, bool tanh_form, int dtype, void *stream) {
    return done(vox_cuda_gelu(x, y, n, tanh_form ? VOX_CUDA_GELU_TANH : VOX_CUDA_GELU_ERF, dtype, stream));
}
VOX_CXX_API bool gpu_snake(const float *x, const float *alpha, const float *beta, float *y, int64_t n, int64_t C, int64_t inner,
                           int kind, void *stream) {
    return done(vox_cuda_snake(x, alpha, beta, y, n, C, inner, kind, stream));
}
VOX_CXX_API bool gpu_bias_add(void *y, const float *b, int64_t rows, int64_t D, int dtype, void *stream) {
    return done(vox_cuda_bias_add(y, b, rows, D, dtype, stream));
}
VOX_CXX_API bool gpu_dequant(bool q4, const void *codes, const void *scale, int scale_dtype, void *out, int out_dtype, int64_t rows,
                             int64_t cols, void *stream) {
    if (q4)
        return done(vox_cuda_dequant_q4(static_cast<const uint8_t *>(codes), scale, scale_dtype, out, out_dtype, rows, cols, stream));
    return done(vox_cuda_dequant_q8(static_cast<const int8_t *>(codes), scale, scale_dtype, out, out_dtype, rows, cols, stream));
}
VOX_CXX_API bool gpu_row_reduce(const void *x, float *out, int64_t rows, int64_t n, int op, int dtype, void *stream) {
    return done(vox_cuda_row_reduce(x, out, rows, n, op, dtype, stream));
}

VOX_CXX_API bool gpu_rope_table(const float *inv_freq, int64_t half, int64_t pos0, int64_t m, float *cs, void *stream) {
    return done(vox_cuda_rope_table(inv_freq, half, pos0, m, cs, stream));
}
VOX_CXX_API bool gpu_qkv_rope(const float *qkv, const float *qn, const float *kn, const float *cs, float *q, float *k_cache,
                              float *v_cache, int64_t m, int64_t heads, int64_t kv_heads, int64_t hd, int64_t pos0, float eps,
                              int64_t ring, void *stream) {
    return done(vox_cuda_qkv_rope(qkv, qn, kn, cs, q, k_cache, v_cache, m, heads, kv_heads, hd, pos0, ring, eps, stream));
}
VOX_CXX_API bool gpu_add_rmsnorm(void *h, const void *delta, const float *layer_scale, const float *w, void *xn, int64_t rows,
                                 int64_t n, float eps, int dtype, void *stream) {
    return done(vox_cuda_add_rmsnorm(h, delta, layer_scale, w, xn, rows, n, eps, dtype, stream));
}
VOX_CXX_API bool gpu_matvec(bool q4, const void *codes, const void *scale, int scale_dtype, const float *bias, const float *x,
                            float *y, int64_t rows, int64_t cols, int64_t m, bool accumulate, void *stream) {
    if (q4)
        return done(vox_cuda_gemv_q4(static_cast<const uint8_t *>(codes), scale, scale_dtype, bias, x, y, rows, cols, m,
                                     accumulate ? 1 : 0, stream));
    return done(vox_cuda_gemv_q8(static_cast<const int8_t *>(codes), scale, scale_dtype, bias, x, y, rows, cols, m,
                                 accumulate ? 1 : 0, stream));
}

// ---- host-pointer conveniences ----

namespace {
// Device scratch for one host call: freed on scope exit.
struct DevBuf {
    void *p = nullptr;
    explicit DevBuf(size_t bytes) { p = gpu_cuda_alloc(bytes); }
    ~DevBuf() { gpu_cuda_free(p); }
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
};
}  // namespace

VOX_CXX_API bool rmsnorm_host(const float *x, const float *w, int64_t rows, int64_t n, float eps, float *out) {
    const size_t xb = size_t(rows) * size_t(n) * 4;
    DevBuf dx(xb), dw(size_t(n) * 4), dy(xb);
    return dx.p && dw.p && dy.p && gpu_cuda_upload(dx.p, x, xb) && gpu_cuda_upload(dw.p, w, size_t(n) * 4) &&
           gpu_rmsnorm(dx.p, static_cast<const float *>(dw.p), rows, n, eps, dy.p) && gpu_cuda_download(out, dy.p, xb) &&
           gpu_cuda_sync();
}

VOX_CXX_API bool softmax_causal_host(const float *scores, float *probs, int64_t heads, int64_t q_len, int64_t n_keys, float scale) {
    const size_t b = size_t(heads) * size_t(q_len) * size_t(n_keys) * 4;
    DevBuf ds(b), dp(b);
    return ds.p && dp.p && gpu_cuda_upload(ds.p, scores, b) &&
           gpu_softmax_causal(static_cast<const float *>(ds.p), static_cast<float *>(dp.p), heads, q_len, n_keys, scale) &&
           gpu_cuda_download(probs, dp.p, b) && gpu_cuda_sync();
}

VOX_CXX_API bool dequant_host(bool q4, const void *codes, const float *scale, int64_t rows, int64_t cols, float *out) {
    const size_t cb = size_t(rows) * size_t(cols) / (q4 ? 2 : 1), sb = size_t(rows) * size_t(cols / 32) * 4,
                 ob = size_t(rows) * size_t(cols) * 4;
    DevBuf dc(cb), ds(sb), dout(ob);
    return dc.p && ds.p && dout.p && gpu_cuda_upload(dc.p, codes, cb) && gpu_cuda_upload(ds.p, scale, sb) &&
           gpu_dequant(q4, dc.p, ds.p, VOX_CUDA_F32, dout.p, VOX_CUDA_F32, rows, cols) && gpu_cuda_download(out, dout.p, ob) &&
           gpu_cuda_sync();
}

}  // namespace vox
