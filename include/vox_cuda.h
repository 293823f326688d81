/*
 * vox_cuda.h — C ABI of the B200 (sm_100a) backend for Vox's memory-bound operator path.
 *
 * Every entry point here replaces an operator of Vox's CPU library (src/kernels.hpp, src/nn.hpp) or an
 * elementwise dispatch of its Vulkan backend (src/gpu_f5.cpp, src/gpu_codec.cpp, src/gpu_vulkan.cpp).
 * The citation above each declaration names the reference interface it stands in for (file:line within
 * the dariumi/Vox project).
 *
 * Conventions (kept from Vox's GPU seam, src/gpu.hpp and src/gpu_vulkan.cpp):
 *   - Return value is a status: 0 = OK, negative = one of the VOX_CUDA_ERR_* codes, whose values equal
 *     Vox's vox_status codes (include/vox.h:48-55). No exception crosses this boundary.
 *   - The message of the last failed call is kept per host thread: vox_cuda_last_error().
 *   - All tensor pointers are DEVICE pointers owned by the caller and never retained after the call (the one
 *     exception: an F5 DiT plan keeps the weight pointers of its description and reads them at every run).
 *   - Every call takes a CUDA stream (cudaStream_t passed as void*, NULL = legacy default stream) and is
 *     asynchronous and stream-ordered. There is no global lock around launches: calls from several host
 *     threads on distinct streams run concurrently.
 *   - There is no CPU fallback. If the device cannot run the kernel the call fails with VOX_CUDA_ERR_DEVICE.
 *   - "Activations" follow the call's dtype (VOX_CUDA_F32 or VOX_CUDA_BF16). Learned weight vectors that Vox
 *     holds as `const float *` (norm weights and biases, Snake alpha/beta) are always f32. Per-batch
 *     modulation vectors of adaLN (shift/scale/gate) follow the call's dtype.
 *   - Arithmetic is f32 for every dtype; bf16 outputs are rounded to nearest-even once, at the store.
 *   - Reductions use a fixed order (no floating-point atomics): results are bitwise reproducible run to run.
 */
#ifndef VOX_CUDA_H
#define VOX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VOX_CUDA_API __attribute__((visibility("default")))
#else
#define VOX_CUDA_API
#endif

/* Status codes: same numeric values as vox_status in include/vox.h:44-56. */
#define VOX_CUDA_OK 0
#define VOX_CUDA_ERR_IO (-1)
#define VOX_CUDA_ERR_FORMAT (-2)
#define VOX_CUDA_ERR_DEVICE (-3)
#define VOX_CUDA_ERR_OOM (-4)
#define VOX_CUDA_ERR_ARG (-6)
#define VOX_CUDA_ERR_UNSUPPORTED (-8)

/* Element types of activations. */
#define VOX_CUDA_F32 0
#define VOX_CUDA_BF16 1
#define VOX_CUDA_F16 2 /* only as a q8/q4 scale type */

/* GELU forms. */
#define VOX_CUDA_GELU_ERF 0  /* 0.5x(1+erf(x/sqrt2)): kernels.hpp:106 gelu_erf, nn.cpp:87-96 gelu_inplace */
#define VOX_CUDA_GELU_TANH 1 /* 0.5x(1+tanh(sqrt(2/pi)(x+0.044715x^3))): f5.cpp:93-96, f5ew.comp mode 1 */

/* Snake forms (all: y = x + coef[c] * s^2 with s = sin(arg[c] * x)). */
#define VOX_CUDA_SNAKE_HIFT 0   /* coef = 1/(alpha+1e-9), arg = alpha, accurate sin: cosyvoice.cpp:239-248 */
#define VOX_CUDA_SNAKE_BETA 1   /* coef = inv_b, arg = a (the precomputed Snake struct): qwen3.cpp:86-94 */
#define VOX_CUDA_SNAKE_KOKORO 2 /* coef = 1/alpha, arg = alpha, Vox's fast_sin polynomial: kokoro.cpp:233-242 */

/* Row reductions. */
#define VOX_CUDA_REDUCE_SUM 0
#define VOX_CUDA_REDUCE_MAX 1
#define VOX_CUDA_REDUCE_L2 2 /* sqrt(sum of squares) */

/* Slot count of the deterministic global sum: lcm(1..8), so every world size 1..8 owns whole slots. */
#define VOX_CUDA_GLOBAL_SUM_SLOTS 840

/* ---------------------------------------------------------------- service */

/* Library version string, e.g. "vox-cuda 0.1.0 sm_100a". */
VOX_CUDA_API const char *vox_cuda_version(void);
/* Message of the last failed call on this host thread ("" if none). Mirrors vox_last_error(), include/vox.h:120. */
VOX_CUDA_API const char *vox_cuda_last_error(void);
/* Number of CUDA devices, written to *count. Mirrors gpu_enumerate(), src/gpu.hpp:35. */
VOX_CUDA_API int vox_cuda_device_count(int *count);
/* Compute capability of the current device as major*10+minor (100 for B200), written to *cc. */
VOX_CUDA_API int vox_cuda_device_cc(int *cc);
/* Device-side error bits of the current device since the last call, written to *flags, then cleared (synchronises
 * with the device). Bit 0 (VOX_CUDA_DEVERR_TIMEOUT): a kernel gave up a bounded wait for its staged data and left
 * its rows unwritten. No counterpart in the reference (Vox's Vulkan backend has no device-side waits). */
#define VOX_CUDA_DEVERR_TIMEOUT 1u
VOX_CUDA_API int vox_cuda_device_error(unsigned int *flags);
/* Test hook of the row operators (RMSNorm, LayerNorm, adaLN, softmax, row reductions, residual + RMSNorm): from the
 * next launch on, the stage barrier of row `row` (-1 = none) expects 16 bytes more than its copies deliver, so every
 * copy lands but the wait for that row runs out after wait_limit_ns (0 = the default 2 s); the warp that owns the row
 * then waits (bounded) for its copies in flight, sets VOX_CUDA_DEVERR_TIMEOUT and stops, leaving that row and its
 * later rows unwritten. Exercises the give-up path without a fault. Call with (-1, 0) to restore normal operation.
 * No counterpart in the reference. */
VOX_CUDA_API int vox_cuda_test_row_stall(int64_t row, uint64_t wait_limit_ns);

/* Seeded synthetic data with Vox's counter-based generator (Philox4x32-10, src/sampling.hpp:16-50).
 * Element i uses counter {i lo, i hi, stream_id, draw}, key {seed lo, seed hi}.
 *   dist 0 = uniform in [a, b): u = (r0 >> 8) * 2^-24 as DetRng::uniform (sampling.hpp:43-46), then a + (b-a)*u.
 *   dist 1 = normal(mean a, std b): Box–Muller on element pairs p = i/2 as F5Model::noise (f5.cpp:402-414).
 *   dist 2 = uniform integer codes in [a, b] (inclusive), written as int8 (dtype ignored): floor(u*(b-a+1)) + a.
 *   dist 3 = uniform bytes (0..255), written as uint8 (dtype ignored): r0 & 0xFF.
 * counter0 offsets the element index, so a shard of a larger tensor draws the same numbers as the whole. */
VOX_CUDA_API int vox_cuda_fill_philox(void *out, int64_t n, int dist, float a, float b, uint64_t seed, uint32_t stream_id,
                                      int64_t counter0, int dtype, void *stream);

/* ---------------------------------------------------------------- normalisation */

/* y[r] = w * (x[r] * 1/sqrt(mean(x[r]^2) + eps)) for r < rows; y may equal x.
 * Replaces vox::rmsnorm(x, w, n, eps, out), src/kernels.hpp:103 (kernels.cpp:707-712), batched over rows;
 * GPU twin of rmsnorm.comp (src/shaders/rmsnorm.comp:1-22). w: f32 [n]. */
VOX_CUDA_API int vox_cuda_rmsnorm(const void *x, const float *w, void *y, int64_t rows, int64_t n, float eps, int dtype,
                                  void *stream);

/* LayerNorm over rows of n. modulate = 0: y = (x-mean)*inv*w + b (w NULL: no scale, b NULL: no shift).
 * modulate = 1: y = (x-mean)*inv*(1+w) + b, the AdaLayerNorm form (w and b required).
 * Replaces vox::layernorm(x, w, b, n, eps, out), src/kernels.hpp:104 (kernels.cpp:714-723), and
 * vox::nn::layer_norm(x, T, C, w, b, eps, modulate), src/nn.hpp:83 (nn.cpp:248-265). y may equal x. */
VOX_CUDA_API int vox_cuda_layernorm(const void *x, const float *w, const float *b, void *y, int64_t rows, int64_t n, float eps,
                                    int modulate, int dtype, void *stream);

/* Fused adaLN block of the F5 DiT over x [B][T][D]:
 *   m = LN(x[b][t]) * (1 + scale[b]) + shift[b]          (LN without affine, eps)
 *   y = residual[b][t] + gate[b] * m                      (gate and residual given)
 *   y = m                                                 (gate and residual NULL: Vox's modulate alone)
 * shift/scale/gate: [B][D] in dtype. Replaces the modulate lambda f5.cpp:617-632 composed with the gated_add
 * lambda f5.cpp:670-676; GPU twin of f5ln.comp mode 1 followed by f5ew.comp mode 0 (gpu_f5.cpp:295,312). */
VOX_CUDA_API int vox_cuda_adaln(const void *x, const void *shift, const void *scale, const void *gate, const void *residual,
                                void *y, int64_t B, int64_t T, int64_t D, float eps, int dtype, void *stream);

/* h[b][t][d] += gate[b][d] * src[b][t][d]; gate [B][D] in dtype.
 * Replaces the gated_add lambda f5.cpp:670-676 (B = 1) and f5ew.comp mode 0 (f5ew.comp:18-19). */
VOX_CUDA_API int vox_cuda_gated_add(void *h, const void *gate, const void *src, int64_t B, int64_t T, int64_t D, int dtype,
                                    void *stream);

/* y[r][o] += b[o] for r < rows, o < D; b: f32 [D].
 * Replaces the bias loop of vox::nn::linear, nn.cpp:148-155 (also Conv/ConvT bias nn.cpp:242-244), f5ew.comp mode 3. */
VOX_CUDA_API int vox_cuda_bias_add(void *y, const float *b, int64_t rows, int64_t D, int dtype, void *stream);

/* ---------------------------------------------------------------- softmax */

/* Scaled row softmax, f32. Row r sees its first `visible` entries: visible = n when q_len == 0, else
 * min(n, (r % q_len) + pos0 + 1) (causal: query i of a head at absolute position pos0+i sees keys 0..pos0+i).
 * y[r][j] = exp(scale*x[r][j] - max) / sum for j < visible, 0 for j >= visible; x beyond visible is not read.
 * y may equal x. Replaces the causal composition kernels.cpp:812-819 around vox::softmax_inplace(x, n),
 * src/kernels.hpp:107 (kernels.cpp:725-732), and the softmax half of attention.comp:20-39. */
VOX_CUDA_API int vox_cuda_softmax_rows(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len,
                                       int64_t pos0, void *stream);

/* ---------------------------------------------------------------- activations */

/* h[i] = silu(g[i]) * u[i], silu(x) = x/(1+exp(-x)); h may equal g.
 * Replaces the SwiGLU loop kernels.cpp:836 over vox::silu, src/kernels.hpp:105; silumul.comp:1-12. */
VOX_CUDA_API int vox_cuda_silu_mul(const void *g, const void *u, void *h, int64_t n, int dtype, void *stream);

/* Fused gate|up layout: gu [m][2I] -> h [m][I] = silu(gu[:, :I]) * gu[:, I:]. Replaces swiglu.comp:1-13. */
VOX_CUDA_API int vox_cuda_swiglu_fused(const void *gu, void *h, int64_t m, int64_t I, int dtype, void *stream);

/* y = gelu(x), kind = VOX_CUDA_GELU_*; y may equal x.
 * Replaces vox::gelu_erf (kernels.hpp:106), vox::nn::gelu_inplace (nn.hpp:125, nn.cpp:87-96), F5's gelu_tanh
 * (f5.cpp:93-96) and f5ew.comp mode 1. */
VOX_CUDA_API int vox_cuda_gelu(const void *x, void *y, int64_t n, int kind, int dtype, void *stream);

/* y = a + b and y = a * b, elementwise (the residual adds of kernels.cpp:830,840 and the sweep ops). */
VOX_CUDA_API int vox_cuda_add(const void *a, const void *b, void *y, int64_t n, int dtype, void *stream);
VOX_CUDA_API int vox_cuda_mul(const void *a, const void *b, void *y, int64_t n, int dtype, void *stream);

/* Snake activation, f32, over n elements whose channel is c = (i / inner) % C:
 *   inner = 1  -> Vox's time-major [T][C] layout;  inner = T -> channel-major [B][C][T].
 * alpha: f32 [C]; beta: f32 [C] for VOX_CUDA_SNAKE_BETA (the Snake struct's inv_b), else NULL. y may equal x.
 * Replaces snake_apply (qwen3.cpp:86-94), SnakeRes::snake (cosyvoice.cpp:239-248), the Kokoro snake
 * (kokoro.cpp:233-242 with fast_sin, nn.hpp:26-40) and snake.comp:1-14. */
VOX_CUDA_API int vox_cuda_snake(const float *x, const float *alpha, const float *beta, float *y, int64_t n, int64_t C,
                                int64_t inner, int kind, void *stream);

/* load_snake (qwen3.cpp:76-84) on the device: a[c] = exp(alpha[c]), inv_b[c] = 1/(exp(beta[c]) + 1e-9). */
VOX_CUDA_API int vox_cuda_snake_beta_params(const float *alpha, const float *beta, float *a, float *inv_b, int64_t C,
                                            void *stream);

/* ---------------------------------------------------------------- block dequantisation */

/* Q8: q int8 [rows][cols], scale [rows][cols/32] (scale_dtype VOX_CUDA_F32 = Vox's layout, or VOX_CUDA_F16);
 * out[r][k] = float(q[r][k]) * scale[r][k/32], written as out_dtype (VOX_CUDA_F32 or VOX_CUDA_BF16, RNE).
 * cols % 32 == 0. Bit-exact with vox::mat_row / mat_gather (kernels.cpp:446-452,468-471), Mat layout kernels.hpp:45. */
VOX_CUDA_API int vox_cuda_dequant_q8(const int8_t *q, const void *scale, int scale_dtype, void *out, int out_dtype, int64_t rows,
                                     int64_t cols, void *stream);

/* Q4: packed [rows][cols/2] bytes, 16 bytes per 32-weight block; byte j of a block holds element j in its low nibble
 * and element j+16 in its high nibble; value = (code - 8) * scale. Layout kernels.hpp:46-47, bit-exact with
 * vox::mat_row Q4 (kernels.cpp:453-463). */
VOX_CUDA_API int vox_cuda_dequant_q4(const uint8_t *q, const void *scale, int scale_dtype, void *out, int out_dtype, int64_t rows,
                                     int64_t cols, void *stream);

/* ---------------------------------------------------------------- reductions */

/* out[r] = sum / max / sqrt(sum of squares) of row r of x [rows][n], f32 result.
 * No single reference function: the same reductions sit inside vox::rmsnorm (kernels.cpp:709) and
 * vox::softmax_inplace (kernels.cpp:727-729). Fixed order: lane l of a warp takes 4-wide vectors l, l+32, ...
 * of the row, keeps one accumulator per vector component, folds them as (c0+c1)+(c2+c3) and the 32 lanes by an
 * xor butterfly (16, 8, 4, 2, 1). */
VOX_CUDA_API int vox_cuda_row_reduce(const void *x, float *out, int64_t rows, int64_t n, int op, int dtype, void *stream);

/* Deterministic global sum across shards, step 1 of 2 (no reference counterpart: Vox has no multi-device code).
 * The global tensor has total_rows rows of n; this shard holds rows [row0, row0 + rows). Slot s of
 * VOX_CUDA_GLOBAL_SUM_SLOTS covers global rows [floor(s*R/S), floor((s+1)*R/S)). The shard's rows must be a whole
 * number of slots. Writes slots[S] (f64): each owned slot = fixed-order sum of its row sums, every other slot 0.
 * rowsum_scratch: device f32 [rows], caller-allocated scratch for the row sums.
 * Summing the slot vectors of all shards element-wise (one NCCL all-reduce) is exact (x + 0 = x), so step 2 gives
 * a result that is bitwise identical for any number of shards. */
VOX_CUDA_API int vox_cuda_global_sum_partials(const void *x, int64_t rows, int64_t n, int64_t row0, int64_t total_rows,
                                              float *rowsum_scratch, double *slots, int dtype, void *stream);

/* Step 2: out[0] = fixed-order pairwise sum of slots[VOX_CUDA_GLOBAL_SUM_SLOTS] (f64). */
VOX_CUDA_API int vox_cuda_global_sum_finish(const double *slots, double *out, void *stream);

/* Global sum of a whole single-device tensor x [rows][n] into out[0] (f64) without any allocation: the same kernels
 * and result as vox_cuda_global_sum_partials (row0 = 0, total_rows = rows) followed by vox_cuda_global_sum_finish,
 * with the row sums and slots kept in a fixed scratch array inside the library instead of caller memory. For callers
 * that cannot call cudaMalloc (a real-time audio callback, where an allocation can block and synchronise the device;
 * a plugin host that owns all device memory apart from the inputs and outputs it passes in).
 * Limit: rows <= 262144 (larger tensors are rejected with VOX_CUDA_ERR_ARG). The scratch array (about 1 MB) lives in
 * the library's device module: it is held on every device where that module is loaded until the process exits (with
 * CUDA's lazy module loading, from the library's first use on that device, at the latest this entry point's first
 * call there). The first call in each CUDA context looks up the array's device address (cudaGetSymbolAddress) and may
 * load the module and block: make it a warm-up call outside the real-time path, before any stream capture, on every
 * device. A new context of the device (after cudaDeviceReset) is detected and its address looked up again. All calls
 * share the one array, so calls whose kernels overlap on the GPU (different streams without ordering) race; order them.
 * No counterpart in the reference (Vox has no device-side global sum). */
VOX_CUDA_API int vox_cuda_global_sum_noalloc(const void *x, int64_t rows, int64_t n, double *out, int dtype, void *stream);

/* Cross-GPU global sum in one call. A communicator spans the shards (one rank per GPU; NCCL, loaded at run time):
 *   vox_cuda_comm_unique_id   rank 0 draws the id (VOX_CUDA_COMM_ID_BYTES bytes) and hands it to every rank;
 *   vox_cuda_comm_init_rank   each process joins with it (non-blocking communicator; fails with VOX_CUDA_ERR_DEVICE if
 *                             not every rank joined within timeout_ms, 0 = 30 s);
 *   vox_cuda_comm_init_all    one process driving ndev GPUs gets one communicator per device;
 *   vox_cuda_comm_wait        waits (host polling) until the stream's work is done; past timeout_ms (0 = 30 s), or on an
 *                             NCCL error, the communicator is aborted (its kernels end) and VOX_CUDA_ERR_DEVICE returned:
 *                             a lost peer is reported to the host instead of hanging;
 *   vox_cuda_comm_destroy.
 * vox_cuda_global_sum = vox_cuda_global_sum_partials of this shard (rows [row0, row0 + rows) of the [total_rows][n]
 * global tensor), then one all-reduce of the 840 f64 slots over comm (comm NULL or of one rank: none), then
 * vox_cuda_global_sum_finish into out[0]; every rank gets the same bits for any number of ranks 1..8. Stream-ordered;
 * rowsum_scratch: f32 [rows], slots: f64 [840] (device). With vox_cuda_comm_init_all, wrap the ndev calls (one per
 * device, each with that device current) in vox_cuda_comm_group_start / _end.
 * No counterpart in the reference (Vox drives one device per process and has no global reduction). */
#define VOX_CUDA_COMM_ID_BYTES 128
typedef struct vox_cuda_comm vox_cuda_comm;
VOX_CUDA_API int vox_cuda_comm_unique_id(void *id);
VOX_CUDA_API int vox_cuda_comm_init_rank(const void *id, int nranks, int rank, int timeout_ms, vox_cuda_comm **out);
VOX_CUDA_API int vox_cuda_comm_init_all(int ndev, const int *devices, vox_cuda_comm **comms);
VOX_CUDA_API int vox_cuda_comm_group_start(void);
VOX_CUDA_API int vox_cuda_comm_group_end(void);
VOX_CUDA_API int vox_cuda_comm_wait(vox_cuda_comm *comm, void *stream, int timeout_ms);
VOX_CUDA_API void vox_cuda_comm_destroy(vox_cuda_comm *comm);
VOX_CUDA_API int vox_cuda_global_sum(const void *x, int64_t rows, int64_t n, int64_t row0, int64_t total_rows, float *rowsum_scratch,
                                     double *slots, double *out, int dtype, vox_cuda_comm *comm, void *stream);

/* ---------------------------------------------------------------- transformer elementwise chain */

/* RoPE table for m positions pos0 .. pos0+m-1: cs[(i*half + p)*2] = cos(f), cs[(i*half + p)*2 + 1] = sin(f),
 * f = inv_freq[p] * float(pos0 + i) in f32 (cs: f32 [m][half][2], 8-byte aligned; inv_freq: f32 [half], e.g. from
 * vox::rope_inv_freq, kernels.cpp:734-738). Replaces the host loop that fills the GPU transformer's table
 * (gpu_vulkan.cpp:855-860) and the cos/sin part of vox::rope_apply (kernels.cpp:744-747). One table serves every
 * layer of a forward pass. cos/sin are CUDA's sincosf: within 2 ulp of libm's cosf/sinf. */
VOX_CUDA_API int vox_cuda_rope_table(const float *inv_freq, int64_t half, int64_t pos0, int64_t m, float *cs, void *stream);

/* One layer's QKV split + q/k head RMSNorm + RoPE + K/V cache write for m tokens at positions pos0 .. pos0+m-1.
 *   qkv:  f32 [m][heads*hd + 2*kv_heads*hd], the fused projection: q heads, then k heads, then v heads
 *   q:    f32 [m][heads*hd]                                   <- rope(headnorm_q(q part))
 *   k_cache, v_cache: f32 [rows][kv_heads*hd]; token i writes row pos0 + i (ring = 0) or ring slot (pos0 + i) % ring
 *                     (ring > 0 needs m <= ring: no slot is written twice by one call)
 *   q_norm_w / k_norm_w: f32 [hd] RMSNorm weights of the head norms, or NULL for none; eps their epsilon
 *   cs:   the vox_cuda_rope_table rows of these m tokens (row i = position pos0 + i)
 * Rotate-half RoPE: a = x[p], b = x[p + hd/2] -> a*c - b*s, b*c + a*s. Replaces shaders/qkvsplit.comp:10-19,
 * shaders/qkrope.comp:11-33 (run over q and over the K cache rows, gpu_vulkan.cpp:686-698) and shaders/ringput.comp;
 * CPU form transformer_forward kernels.cpp:797-806 (vox::rmsnorm per head, vox::rope_apply kernels.cpp:740-757,
 * appends to the KV cache). hd even, hd <= 4096; outputs must not overlap qkv. Fast path: hd in {64, 128, 256}
 * with 16-byte aligned buffers. */
VOX_CUDA_API int vox_cuda_qkv_rope(const float *qkv, const float *q_norm_w, const float *k_norm_w, const float *cs, float *q,
                                   float *k_cache, float *v_cache, int64_t m, int64_t heads, int64_t kv_heads, int64_t hd,
                                   int64_t pos0, int64_t ring, float eps, void *stream);

/* Residual update + RMSNorm over rows of n: h[r] += delta[r] * layer_scale (layer_scale f32 [n] or NULL for none),
 * then xn[r] = w * (h[r] * 1/sqrt(mean(h[r]^2) + eps)); h is updated in place, xn must not overlap h or delta.
 * w: f32 [n]. bf16 rows normalise the f32 sum (h stores its bf16 rounding). Replaces transformer_forward's
 * o *= attn_scale; h += o; rmsnorm(h, ln2) (kernels.cpp:822-825, 833) and d *= mlp_scale; h += d before the next
 * layer's rmsnorm(h, ln1) (kernels.cpp:829-831, 793); on Vox's GPU the accumulating GEMM epilogue followed by
 * rmsnorm.comp (gpu_vulkan.cpp:700-701, 707-708). */
VOX_CUDA_API int vox_cuda_add_rmsnorm(void *h, const void *delta, const float *layer_scale, const float *w, void *xn, int64_t rows,
                                      int64_t n, float eps, int dtype, void *stream);

/* ---------------------------------------------------------------- GEMM on the tensor cores */

/* Activations fused into the GEMM's epilogue. */
#define VOX_CUDA_GEMM_NONE 0
#define VOX_CUDA_GEMM_GELU_ERF 1  /* gemmb.comp flag 2: 0.5 v (1 + erf(v / sqrt 2)) */
#define VOX_CUDA_GEMM_GELU_TANH 2 /* F5's gelu_tanh, f5.cpp:93-96 */

/* y[m][n] = act(x[m][k] . w[n][k]^T + bias[n]): bf16 x and w (row-major, k a multiple of 8, 16-byte aligned), f32
 * accumulation on the 5th-generation tensor cores, y f32 or bf16 (out_dtype); bias f32 [n] or NULL.
 * Replaces the GPU GEMM of Vox's F5 / Vocos linear layers, gemm() in gpu_f5.cpp:287-322 running shaders/gemmb.comp:1-99
 * with its bias (flag 1) and GELU (flag 2) epilogue; the CPU counterpart is vox::matmul with a bias (kernels.cpp:656-706). */
VOX_CUDA_API int vox_cuda_gemm_bf16(const void *x, const void *w, const float *bias, void *y, int64_t m, int64_t n, int64_t k, int act,
                                    int out_dtype, void *stream);

/* ---------------------------------------------------------------- quantized GEMV (decode) */

/* y[i][r] = bias[r] + sum_k W[r][k] * x[i][k] for i < m (accumulate != 0: y[i][r] += that), W[r][k] = code *
 * scale[r][k/32]. Q8: w int8 [rows][cols]; Q4: w uint8 [rows][cols/2], 16 bytes per 32-block, byte j = code j |
 * code j+16 << 4, value (code - 8). scale: [rows][cols/32] in scale_dtype (VOX_CUDA_F32, Vox's layout, or VOX_CUDA_F16);
 * bias f32 [rows] or NULL; x f32 [m][cols]; y f32 [m][rows]. cols % 32 == 0; w and x 16-byte aligned.
 * f32 accuracy (the rounding of an f32 dot product); deterministic. Activation rows are taken 8 per launch, so the
 * weights stream once per 8 rows: this is the decode path (m <= 8 in one pass).
 * Replaces the GPU matvec shaders/matmul.comp:1-178 (rec_mm for m <= 8, gpu_vulkan.cpp:657-674; gpu_matmul
 * gpu_vulkan.cpp:544-572) and, for the CPU, matmul (kernels.cpp:656) with Q8/Q4 weights in its float-activation
 * form (dequantise then f32 product, kernels.cpp:669-688; the Q8 m <= 8 and Q4 CPU paths quantise x to int8 instead,
 * kernels.cpp:498-604). */
VOX_CUDA_API int vox_cuda_gemv_q8(const int8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y,
                                  int64_t rows, int64_t cols, int64_t m, int accumulate, void *stream);
VOX_CUDA_API int vox_cuda_gemv_q4(const uint8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y,
                                  int64_t rows, int64_t cols, int64_t m, int accumulate, void *stream);

/* The prefill form of the same product (many activation rows): y[i][r] (+)= bias[r] + sum_k W[r][k] x[i][k] for i < m,
 * same arguments and weight layouts as vox_cuda_gemv_q8 / q4, on the 5th-generation tensor cores in f16: the weight
 * codes are dequantised to f16 (code * scale, one rounding) and x rounded to f16 once, products accumulated in f32.
 * Error within about 1e-3 of sum |w x| (f16 keeps 11 significant bits); |x| must stay below 65504. Results are
 * identical run to run. Two forms with the same operands: below 256 rows of x one pass (the codes converted inside
 * the GEMM kernel; where the output tiles do not fill the SMs evenly the last wave's tiles are split into K-ranges
 * whose f32 partials are added in a fixed order); from 256 rows two passes (W dequantised to f16 once, then the f16
 * GEMM). Scratch comes from the device's default memory pool, stream-ordered (cudaMallocAsync / cudaFreeAsync on
 * `stream`): m * cols * 2 bytes for x, plus at most 128 KB per SM of partials (one pass) or rows * cols * 2 bytes for
 * the f16 weights (two passes). Replaces, for m > 8, Vox's dequantise-then-f32-matmul path
 * (kernels.cpp:661-688) and its GPU tiled GEMM on q8 weights (shaders/gemmb.comp:1-99 WTYPE 3). */
VOX_CUDA_API int vox_cuda_gemm_q8(const int8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y,
                                  int64_t rows, int64_t cols, int64_t m, int accumulate, void *stream);
VOX_CUDA_API int vox_cuda_gemm_q4(const uint8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y,
                                  int64_t rows, int64_t cols, int64_t m, int accumulate, void *stream);

/* ---------------------------------------------------------------- .tmod weight files -> device */

/* Vox's .tmod container (src/formats.hpp:44-90): 64-byte header "VOXM" v1.x, JSON manifest with a "blobs" table
 * {name: {dtype, shape, offset, nbytes}}, blobs 4096-byte aligned. dtype codes follow Vox's DType order
 * (src/common.hpp:22): F32 0, F16 1, BF16 2, I32 3, I16 4, I8 5, U8 6. */
#define VOX_CUDA_TMOD_MAX_DIMS 8
typedef struct vox_cuda_tmod vox_cuda_tmod;

/* Maps `path` read-only and reads its manifest (the checks and errors of TmodFile::TmodFile, formats.cpp:175-205:
 * VOX_CUDA_ERR_IO for an unreadable file, VOX_CUDA_ERR_FORMAT for a bad header, manifest or blob range). No device
 * work. The handle is not thread-safe for concurrent uploads on different devices. */
VOX_CUDA_API int vox_cuda_tmod_open(const char *path, vox_cuda_tmod **out);
/* Waits for the handle's transfers in flight, frees its staging memory and unmaps the file. NULL is ignored. */
VOX_CUDA_API void vox_cuda_tmod_close(vox_cuda_tmod *t);
/* Number of blobs, their names in manifest order, their description (shape: up to VOX_CUDA_TMOD_MAX_DIMS entries, any
 * output pointer may be NULL), and a host pointer into the mapping (TmodFile::get, formats.cpp:207-211). */
VOX_CUDA_API int vox_cuda_tmod_count(const vox_cuda_tmod *t, int64_t *n);
VOX_CUDA_API int vox_cuda_tmod_name(const vox_cuda_tmod *t, int64_t i, const char **name);
VOX_CUDA_API int vox_cuda_tmod_info(const vox_cuda_tmod *t, const char *name, int *dtype, int64_t *shape, int *ndim,
                                    uint64_t *nbytes);
VOX_CUDA_API int vox_cuda_tmod_data(const vox_cuda_tmod *t, const char *name, const void **host);
/* Copies blobs names[i] into device buffers dst[i] (nbytes each) on `stream`. The first upload page-locks the
 * mapping for the device (read-only registration; blobs then go straight from the page cache); where that is not
 * supported (or VOX_CUDA_TMOD_REGISTER=0) a ring of pinned staging buffers (32 MB x 4) is used, host copies of the next
 * chunk overlapping the transfer of the previous one. Returns when the last copy is queued; the copies complete in
 * stream order (vox_cuda_tmod_close waits for them). Replaces the weight uploads of the Vulkan backend (upload_parts,
 * gpu_vulkan.cpp:476-536). */
VOX_CUDA_API int vox_cuda_tmod_upload(vox_cuda_tmod *t, const char *const *names, int64_t count, void *const *dst, void *stream);
/* Uploads the Q8 (I8) or Q4 (U8, two codes per byte) matrix `name` and its "<name>.scale" f32 blob as nn::mat_named
 * reads them (nn.cpp:132-145) and dequantises it on the device into dst [rows][cols] (out_dtype F32 or BF16),
 * bit-exact with mat_row (kernels.cpp:446-463). Device staging comes from the stream-ordered allocator. */
VOX_CUDA_API int vox_cuda_tmod_upload_dequant(vox_cuda_tmod *t, const char *name, void *dst, int out_dtype, void *stream);

/* ---------------------------------------------------------------- F5 DiT step (one CUDA graph) */

/* One F5-TTS DiT step as the Vulkan backend records it (gpu_f5_step, gpu_f5.cpp:273-332) and the CPU computes it
 * (F5Model::dit_forward, f5.cpp:563-724). Input embedding (when in_proj is given): h = [x, cond, temb] . W_in^T + b
 * per row, then per sequence h += mish(conv2(mish(conv1(h)))), two grouped (16) 1-D convolutions over time of kernel
 * 31 with zero padding (Conv1d::forward, f5_ops.cpp:106-145; mish f5.cpp:97-100). Per block: ada = W_ada . ts ([shift,
 * scale, gate] of attention, then of the MLP); nrm = LayerNorm(h) (no affine, eps 1e-6) * (1 + scale) + shift;
 * q, k, v = nrm . W^T; RoPE on interleaved pairs (2j, 2j+1) at the frame position, on the first pe_attn_head heads
 * (all heads if 0); attention without mask per sequence and head, softmax(q k^T / sqrt(dim_head)) v;
 * h += gate_msa * (at . W_o^T); the MLP the same way with GELU (tanh form) between ff1 and ff2. Output:
 * fin = W_norm_out . ts = [scale, shift], out = (LayerNorm(h) * (1 + scale) + shift) . W_proj^T.
 * Every linear layer is y = x W^T + b as Vox's matmul computes it (kernels.hpp:83, the bias a Mat carries when the
 * file holds "<name>.bias", f5.cpp:59-84); a NULL bias is zero. Weights and biases are f32 device buffers, weights
 * [out][in] (Vox's Mat layout; convolutions [dim][dim/16][31] as PyTorch stores them), owned by the caller and read at
 * every run (the bf16 mode reads its own bf16 copies of the q, k, v, o, ff1, ff2 and proj_out weights, made at create,
 * and its own f32 copies of the biases; the convolution weights are reordered into a copy at create). ts is the
 * SiLU'd time embedding (F5Model::time_embed, f5.cpp:510-526), computed by the caller. */
#define VOX_CUDA_F5_MATH_F32 0  /* f32 GEMMs on the CUDA cores (reference accuracy) */
#define VOX_CUDA_F5_MATH_TF32 1 /* tensor cores, TF32 inputs, f32 accumulation */
#define VOX_CUDA_F5_MATH_BF16 2 /* tensor cores, bf16 inputs, f32 accumulation; with dim_head 64 (and dim % 4 == 0,
                                 * dim <= 2048) the plan snapshots bf16 copies of the projection weights at create, feeds
                                 * every GEMM bf16 activations and runs attention as one fused kernel (scores never leave
                                 * the SM); otherwise cuBLAS may keep the f32 inputs in TF32 */
typedef struct vox_cuda_f5_block_weights {
    const float *ada;        /* [6 dim][dim] */
    const float *q, *k, *v;  /* [heads * dim_head][dim] */
    const float *o;          /* [dim][heads * dim_head] */
    const float *ff1;        /* [ff_mult * dim][dim] */
    const float *ff2;        /* [dim][ff_mult * dim] */
    const float *ada_b, *q_b, *k_b, *v_b, *o_b, *ff1_b, *ff2_b; /* biases [out] of the same layers, or NULL */
} vox_cuda_f5_block_weights;
typedef struct vox_cuda_f5_desc {
    int32_t dim, heads, dim_head, ff_mult, depth, pe_attn_head, out_dim;
    int32_t batch, frames;  /* the step processes batch sequences of `frames` rows each */
    int32_t math;           /* VOX_CUDA_F5_MATH_* */
    const vox_cuda_f5_block_weights *blocks; /* [depth], copied at create */
    const float *norm_out;  /* [2 dim][dim]: (scale, shift) */
    const float *proj_out;  /* [out_dim][dim] */
    const float *norm_out_b, *proj_out_b; /* their biases, or NULL */
    /* input embedding, or in_proj NULL (the caller writes h): x [rows][out_dim] and cond [rows][in_dim - out_dim]
     * (the condition mel then the text embedding) form the in_dim-wide input rows */
    int32_t in_dim;
    const float *in_proj, *in_proj_b;                /* [dim][in_dim], [dim] */
    const float *pos1_w, *pos1_b, *pos2_w, *pos2_b;  /* [dim][dim/16][31], [dim] */
} vox_cuda_f5_desc;
typedef struct vox_cuda_f5 vox_cuda_f5;
/* Allocates the plan's buffers on the current device (h [batch*frames][dim], ts [dim], out [batch*frames][out_dim] and
 * the intermediates), builds the RoPE table as the CPU does (f5.cpp:529-541), runs the step once on `stream` and
 * captures it into a CUDA graph. */
VOX_CUDA_API int vox_cuda_f5_create(const vox_cuda_f5_desc *desc, void *stream, vox_cuda_f5 **out);
/* The plan's device buffers: the caller writes ts and either h (no embedding) or x and cond (embedding; x changes every
 * step, cond stays for a sequence) before a run, and reads out (and the final h) after it. x and cond are NULL without
 * an embedding. */
VOX_CUDA_API int vox_cuda_f5_buffers(vox_cuda_f5 *p, float **h, float **ts, float **out);
VOX_CUDA_API int vox_cuda_f5_inputs(vox_cuda_f5 *p, float **x, float **cond);
/* Replays the captured step on `stream` (stream-ordered, asynchronous). */
VOX_CUDA_API int vox_cuda_f5_run(vox_cuda_f5 *p, void *stream);
/* Frees the plan (waits for its work). NULL is ignored. */
VOX_CUDA_API void vox_cuda_f5_destroy(vox_cuda_f5 *p);

#ifdef __cplusplus
}
#endif

#endif /* VOX_CUDA_H */
