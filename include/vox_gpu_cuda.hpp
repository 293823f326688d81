// vox_gpu_cuda.hpp — the C++17 host seam of the B200 backend, in the style of Vox's src/gpu.hpp.
//
// Vox's in-tree callers (src/kernels.cpp, src/nn.cpp, the model files) use a backend-neutral GPU seam whose calls
// return bool, never throw, and leave the reason of a failure in GpuStats::last_error (src/gpu.hpp:10-17,
// gpu_vulkan.cpp:531-535). This header gives the same seam for the CUDA backend on top of the C ABI
// (include/vox_cuda.h): one batched call per operator of Vox's operator API (src/kernels.hpp:103-107,
// src/nn.hpp:83,125-127) on device pointers, plus host-pointer conveniences that copy in, run and copy out, for
// callers that hold their tensors in host memory as Vox's CPU code does.
//
// Thread safety follows gpu_vulkan.cpp's model without its global lock around recording: a mutex guards only
// device initialisation; launches are stream-ordered and may come from several threads on distinct streams.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include "vox_cuda.h"

namespace vox {

// Call accounting, as GpuStats (src/gpu.hpp:16): successes, failures and the last failure's message.
struct GpuCudaStats {
    int64_t calls_ok = 0, calls_failed = 0;
    std::string last_error;
};

// Selects CUDA device `device` for this thread (gpu_init, src/gpu.hpp:11). false (reason in err) if the device is
// missing or is not an sm_100 part.
bool gpu_cuda_init(int device, std::string &err);
bool gpu_cuda_active();
std::string gpu_cuda_device_name();
GpuCudaStats gpu_cuda_stats();

// Device memory for callers that have no allocator of their own (the uploads of gpu_upload, src/gpu.hpp:14).
void *gpu_cuda_alloc(size_t bytes);
void gpu_cuda_free(void *p);
bool gpu_cuda_upload(void *dst, const void *src, size_t bytes, void *stream = nullptr);
bool gpu_cuda_download(void *dst, const void *src, size_t bytes, void *stream = nullptr);
bool gpu_cuda_sync(void *stream = nullptr);

// ---- device-pointer operators (dtype: VOX_CUDA_F32 or VOX_CUDA_BF16 activations) ----

// vox::rmsnorm (kernels.hpp:103) over rows.
bool gpu_rmsnorm(const void *x, const float *w, int64_t rows, int64_t n, float eps, void *out, int dtype = VOX_CUDA_F32,
                 void *stream = nullptr);
// vox::layernorm (kernels.hpp:104) over rows; b may be NULL.
bool gpu_layernorm(const void *x, const float *w, const float *b, int64_t rows, int64_t n, float eps, void *out,
                   int dtype = VOX_CUDA_F32, void *stream = nullptr);
// vox::nn::layer_norm (nn.hpp:83), in place on x [T][C].
bool gpu_layer_norm(void *x, int T, int C, const float *w, const float *b, float eps, bool modulate, int dtype = VOX_CUDA_F32,
                    void *stream = nullptr);
// F5 adaLN block: modulate (f5.cpp:617-632), then gated residual (f5.cpp:670-676) when gate/residual are given.
bool gpu_adaln(const void *x, const void *shift, const void *scale, const void *gate, const void *residual, void *out, int64_t B,
               int64_t T, int64_t D, float eps = 1e-6f, int dtype = VOX_CUDA_F32, void *stream = nullptr);
// Scaled causal softmax of attention scores [heads][q_len][n_keys] (kernels.cpp:812-819).
bool gpu_softmax_causal(const float *scores, float *probs, int64_t heads, int64_t q_len, int64_t n_keys, float scale,
                        int64_t pos0 = 0, void *stream = nullptr);
// SwiGLU g = silu(g) * u (kernels.cpp:836).
bool gpu_silu_mul(const void *g, const void *u, void *h, int64_t n, int dtype = VOX_CUDA_F32, void *stream = nullptr);
// vox::nn::gelu_inplace (nn.hpp:125) / gelu_erf (kernels.hpp:106) / F5 gelu_tanh (f5.cpp:93-96).
bool gpu_gelu(const void *x, void *y, int64_t n, bool tanh_form = false, int dtype = VOX_CUDA_F32, void *stream = nullptr);
// Snake over time-major x [T][C] (Vox's layout) or channel-major [B][C][T] (inner = T); kind = VOX_CUDA_SNAKE_*.
bool gpu_snake(const float *x, const float *alpha, const float *beta, float *y, int64_t n, int64_t C, int64_t inner, int kind,
               void *stream = nullptr);
// vox::nn::linear's bias add (nn.cpp:151-154): y [rows][D] += b.
bool gpu_bias_add(void *y, const float *b, int64_t rows, int64_t D, int dtype = VOX_CUDA_F32, void *stream = nullptr);
// mat_gather of every row of a Q8 / Q4 matrix (kernels.cpp:446-471); q4 selects the packed 4-bit layout.
bool gpu_dequant(bool q4, const void *codes, const void *scale, int scale_dtype, void *out, int out_dtype, int64_t rows,
                 int64_t cols, void *stream = nullptr);
// Row sum / max / L2 norm (op = VOX_CUDA_REDUCE_*), f32 results.
bool gpu_row_reduce(const void *x, float *out, int64_t rows, int64_t n, int op, int dtype = VOX_CUDA_F32, void *stream = nullptr);

// ---- transformer chain and decode matvec (transformer_forward, kernels.cpp:793-833; rec_layers, gpu_vulkan.cpp:679-715) ----
// cos/sin table of positions pos0 .. pos0+m-1 (gpu_vulkan.cpp:855-860), once per forward for all layers.
bool gpu_rope_table(const float *inv_freq, int64_t half, int64_t pos0, int64_t m, float *cs, void *stream = nullptr);
// One layer's QKV split + q/k head RMSNorm (qn/kn may be NULL) + RoPE + K/V cache write (qkvsplit.comp, qkrope.comp).
bool gpu_qkv_rope(const float *qkv, const float *qn, const float *kn, const float *cs, float *q, float *k_cache, float *v_cache,
                  int64_t m, int64_t heads, int64_t kv_heads, int64_t hd, int64_t pos0, float eps, int64_t ring = 0,
                  void *stream = nullptr);
// h += delta (* layer_scale), xn = rmsnorm(h) (kernels.cpp:822-825, 833).
bool gpu_add_rmsnorm(void *h, const void *delta, const float *layer_scale, const float *w, void *xn, int64_t rows, int64_t n, float eps,
                     int dtype = VOX_CUDA_F32, void *stream = nullptr);
// y [m][rows] (+)= W x for Q8 / Q4 weights (q4 selects the packed layout), f32 activations: gpu_matmul's m <= 8 path
// (gpu_vulkan.cpp:544-572, matmul.comp). bias may be NULL.
bool gpu_matvec(bool q4, const void *codes, const void *scale, int scale_dtype, const float *bias, const float *x, float *y,
                int64_t rows, int64_t cols, int64_t m, bool accumulate = false, void *stream = nullptr);

// ---- host-pointer conveniences (copy in, run, copy out; synchronous) ----
bool rmsnorm_host(const float *x, const float *w, int64_t rows, int64_t n, float eps, float *out);
bool softmax_causal_host(const float *scores, float *probs, int64_t heads, int64_t q_len, int64_t n_keys, float scale);
bool dequant_host(bool q4, const void *codes, const float *scale, int64_t rows, int64_t cols, float *out);

}  // namespace vox
