// F5-TTS DiT step on the device, captured as one CUDA graph (vox_cuda_f5_*).
//
// The step is the transformer half of Vox's gpu_f5_step (gpu_f5.cpp:273-332; CPU F5Model::dit, f5.cpp:608-724): for
// each block an ada GEMV, the modulated LayerNorm, the q/k/v projections, RoPE, unmasked attention per sequence and
// head, the output projection and gated residual, then the MLP (ff1, GELU-tanh, ff2) and its gated residual; at the
// end the final modulation and the output projection. The elementwise and normalisation steps are this library's
// kernels (vox_cuda_adaln with no gate, vox_cuda_gated_add, vox_cuda_gelu, vox_cuda_softmax_rows) plus the RoPE kernel
// below; the projections and the two attention products are cuBLAS GEMMs (f32, or on the tensor cores with TF32 or
// bf16 inputs and f32 accumulation). Attention materialises the score matrix of one sequence at a time
// ([heads][frames][frames] f32) and normalises it in place with the row softmax.
//
// The plan records the whole step once eagerly (kernel selection, first-use attributes), then again under stream
// capture; a run is one cudaGraphLaunch. All buffers are the plan's, so the graph's pointers never change.
#include <cublas_v2.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "common.cuh"

namespace voxcuda {
namespace {

// RoPE on interleaved pairs (2j, 2j+1), in place on q and k [rows][inner]: row r is at position r % frames; heads
// 0 .. rope_heads-1 rotate. cs [frames][half] holds (cos, sin). Each product and sum rounded separately, as the CPU
// loop computes it (f5.cpp:696-701): x0 c - x1 s, x1 c + x0 s.
__global__ void __launch_bounds__(256) f5_rope_kernel(float *q, float *k, const float2 *cs, uint32_t pairs, uint32_t frames,
                                                      uint32_t half, uint32_t rope_heads, uint32_t hd, uint32_t inner) {
    pdl_enter();
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += stride) {
        const uint32_t j = i % half, t = i / half;
        const uint32_t h = t % rope_heads, r = t / rope_heads;
        const float2 c = cs[size_t(r % frames) * half + j];
        const size_t off = size_t(r) * inner + size_t(h) * hd + 2 * j;
        float2 *pq = reinterpret_cast<float2 *>(q + off), *pk = reinterpret_cast<float2 *>(k + off);
        const float2 a = *pq, b = *pk;
        *pq = make_float2(__fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(a.y, c.y)), __fadd_rn(__fmul_rn(a.y, c.x), __fmul_rn(a.x, c.y)));
        *pk = make_float2(__fsub_rn(__fmul_rn(b.x, c.x), __fmul_rn(b.y, c.y)), __fadd_rn(__fmul_rn(b.y, c.x), __fmul_rn(b.x, c.y)));
    }
}

const char *blas_name(cublasStatus_t s) {
    switch (s) {
        case CUBLAS_STATUS_NOT_INITIALIZED: return "not initialized";
        case CUBLAS_STATUS_ALLOC_FAILED: return "allocation failed";
        case CUBLAS_STATUS_INVALID_VALUE: return "invalid value";
        case CUBLAS_STATUS_ARCH_MISMATCH: return "architecture mismatch";
        case CUBLAS_STATUS_EXECUTION_FAILED: return "execution failed";
        case CUBLAS_STATUS_NOT_SUPPORTED: return "not supported";
        default: return "error";
    }
}

}  // namespace

struct F5Plan {
    vox_cuda_f5_desc d{};
    std::vector<vox_cuda_f5_block_weights> blocks;
    int64_t R = 0, inner = 0, ff = 0;
    cublasHandle_t blas = nullptr;
    cublasComputeType_t compute = CUBLAS_COMPUTE_32F_PEDANTIC;
    cudaStream_t cap = nullptr;  // private stream the graph is captured on
    void *ws = nullptr;
    float *h = nullptr, *ts = nullptr, *out = nullptr, *nrm = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *at = nullptr,
          *o = nullptr, *ffb = nullptr, *s = nullptr, *ada = nullptr, *fin = nullptr;
    float2 *cs = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {

constexpr size_t kBlasWorkspace = size_t(32) << 20;

int blas_check(cublasStatus_t s, const char *what) {
    if (s == CUBLAS_STATUS_SUCCESS) return VOX_CUDA_OK;
    return set_error(VOX_CUDA_ERR_DEVICE, std::string("vox_cuda_f5: cuBLAS ") + what + ": " + blas_name(s));
}

// y[R][O] = x[R][I] . W[O][I]^T, all row-major (column-major y^T = op_T(W^T) . x^T).
int gemm_xwt(F5Plan &p, const float *x, const float *w, float *y, int64_t R, int64_t O, int64_t I) {
    const float one = 1.0f, zero = 0.0f;
    return blas_check(cublasGemmEx(p.blas, CUBLAS_OP_T, CUBLAS_OP_N, int(O), int(R), int(I), &one, w, CUDA_R_32F, int(I), x,
                                   CUDA_R_32F, int(I), &zero, y, CUDA_R_32F, int(O), p.compute, CUBLAS_GEMM_DEFAULT),
                      "gemm");
}

#define F5_TRY(expr)                          \
    do {                                      \
        const int rc_ = (expr);               \
        if (rc_ != VOX_CUDA_OK) return rc_;   \
    } while (0)

// Unmasked attention of sequence b: S_h = q_h k_h^T (per head, [frames][frames]), softmax(S_h / sqrt(hd)) in place,
// at_h = P_h v_h. Head h of row i sits at column h * hd of the [rows][inner] tensors.
int attention(F5Plan &p, int64_t b, cudaStream_t st) {
    const int N = p.d.frames, HD = p.d.dim_head, H = p.d.heads, IN = int(p.inner);
    const size_t base = size_t(b) * size_t(N) * size_t(IN);
    const float one = 1.0f, zero = 0.0f;
    // column-major C (j, i) = sum_d K(j, d) Q(i, d): S[i][j] row-major
    F5_TRY(blas_check(cublasGemmStridedBatchedEx(p.blas, CUBLAS_OP_T, CUBLAS_OP_N, N, N, HD, &one, p.k + base, CUDA_R_32F, IN, HD,
                                                 p.q + base, CUDA_R_32F, IN, HD, &zero, p.s, CUDA_R_32F, N, int64_t(N) * N, H,
                                                 p.compute, CUBLAS_GEMM_DEFAULT),
                      "scores"));
    F5_TRY(vox_cuda_softmax_rows(p.s, p.s, int64_t(H) * N, N, 1.0f / std::sqrt(float(HD)), 0, 0, st));
    // column-major C (d, i) = sum_j V(j, d) P[i][j]: at[i][h hd + d]
    return blas_check(cublasGemmStridedBatchedEx(p.blas, CUBLAS_OP_N, CUBLAS_OP_N, HD, N, N, &one, p.v + base, CUDA_R_32F, IN, HD,
                                                 p.s, CUDA_R_32F, N, int64_t(N) * N, &zero, p.at + base, CUDA_R_32F, IN, HD, H,
                                                 p.compute, CUBLAS_GEMM_DEFAULT),
                      "attention output");
}

// The whole step on stream st (eager or under capture; cuBLAS is bound to the same stream).
int record(F5Plan &p, cudaStream_t st) {
    const vox_cuda_f5_desc &d = p.d;
    const int64_t R = p.R, D = d.dim, IN = p.inner, FF = p.ff;
    const uint32_t rope_heads = uint32_t(d.pe_attn_head > 0 ? d.pe_attn_head : d.heads);
    const uint32_t half = uint32_t(d.dim_head / 2);
    const uint32_t pairs = uint32_t(R) * rope_heads * half;
    const int rope_grid = grid_for(pairs, 256, 4);
    for (const vox_cuda_f5_block_weights &L : p.blocks) {
        F5_TRY(gemm_xwt(p, p.ts, L.ada, p.ada, 1, 6 * D, D));
        const float *shift_msa = p.ada, *scale_msa = p.ada + D, *gate_msa = p.ada + 2 * D;
        const float *shift_mlp = p.ada + 3 * D, *scale_mlp = p.ada + 4 * D, *gate_mlp = p.ada + 5 * D;
        F5_TRY(vox_cuda_adaln(p.h, shift_msa, scale_msa, nullptr, nullptr, p.nrm, 1, R, D, 1e-6f, VOX_CUDA_F32, st));
        F5_TRY(gemm_xwt(p, p.nrm, L.q, p.q, R, IN, D));
        F5_TRY(gemm_xwt(p, p.nrm, L.k, p.k, R, IN, D));
        F5_TRY(gemm_xwt(p, p.nrm, L.v, p.v, R, IN, D));
        launch_k(f5_rope_kernel, rope_grid, 256, 0, st, p.q, p.k, (const float2 *)p.cs, pairs, uint32_t(d.frames), half, rope_heads,
                 uint32_t(d.dim_head), uint32_t(IN));
        F5_TRY(check_launch("vox_cuda_f5 rope"));
        for (int64_t b = 0; b < d.batch; ++b) F5_TRY(attention(p, b, st));
        F5_TRY(gemm_xwt(p, p.at, L.o, p.o, R, D, IN));
        F5_TRY(vox_cuda_gated_add(p.h, gate_msa, p.o, 1, R, D, VOX_CUDA_F32, st));
        F5_TRY(vox_cuda_adaln(p.h, shift_mlp, scale_mlp, nullptr, nullptr, p.nrm, 1, R, D, 1e-6f, VOX_CUDA_F32, st));
        F5_TRY(gemm_xwt(p, p.nrm, L.ff1, p.ffb, R, FF, D));
        F5_TRY(vox_cuda_gelu(p.ffb, p.ffb, R * FF, VOX_CUDA_GELU_TANH, VOX_CUDA_F32, st));
        F5_TRY(gemm_xwt(p, p.ffb, L.ff2, p.o, R, D, FF));
        F5_TRY(vox_cuda_gated_add(p.h, gate_mlp, p.o, 1, R, D, VOX_CUDA_F32, st));
    }
    F5_TRY(gemm_xwt(p, p.ts, d.norm_out, p.fin, 1, 2 * D, D));  // fin = [scale, shift] (f5.cpp:720-722)
    F5_TRY(vox_cuda_adaln(p.h, p.fin + D, p.fin, nullptr, nullptr, p.nrm, 1, R, D, 1e-6f, VOX_CUDA_F32, st));
    return gemm_xwt(p, p.nrm, d.proj_out, p.out, R, d.out_dim, D);
}

void release(F5Plan *p) {
    if (!p) return;
    if (p->cap) cudaStreamSynchronize(p->cap);
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    if (p->blas) cublasDestroy(p->blas);
    for (void *b : {(void *)p->ws, (void *)p->h, (void *)p->ts, (void *)p->out, (void *)p->nrm, (void *)p->q, (void *)p->k,
                    (void *)p->v, (void *)p->at, (void *)p->o, (void *)p->ffb, (void *)p->s, (void *)p->ada, (void *)p->fin,
                    (void *)p->cs})
        if (b) cudaFree(b);
    if (p->cap) cudaStreamDestroy(p->cap);
    delete p;
}

template <class T> int alloc(T **ptr, size_t count, const char *what) {
    if (cudaMalloc(reinterpret_cast<void **>(ptr), count * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return set_error(VOX_CUDA_ERR_OOM, std::string("vox_cuda_f5_create: cannot allocate ") + what);
    }
    return VOX_CUDA_OK;
}

int build(F5Plan &p, cudaStream_t user) {
    const vox_cuda_f5_desc &d = p.d;
    const size_t R = size_t(p.R), D = size_t(d.dim), IN = size_t(p.inner), FF = size_t(p.ff), N = size_t(d.frames);
    F5_TRY(alloc(&p.h, R * D, "h"));
    F5_TRY(alloc(&p.ts, D, "ts"));
    F5_TRY(alloc(&p.out, R * size_t(d.out_dim), "out"));
    F5_TRY(alloc(&p.nrm, R * D, "nrm"));
    F5_TRY(alloc(&p.q, R * IN, "q"));
    F5_TRY(alloc(&p.k, R * IN, "k"));
    F5_TRY(alloc(&p.v, R * IN, "v"));
    F5_TRY(alloc(&p.at, R * IN, "at"));
    F5_TRY(alloc(&p.o, R * D, "o"));
    F5_TRY(alloc(&p.ffb, R * FF, "ff"));
    F5_TRY(alloc(&p.s, size_t(d.heads) * N * N, "scores"));
    F5_TRY(alloc(&p.ada, 6 * D, "ada"));
    F5_TRY(alloc(&p.fin, 2 * D, "fin"));
    F5_TRY(alloc(&p.cs, N * size_t(d.dim_head / 2), "rope table"));
    F5_TRY(alloc(reinterpret_cast<uint8_t **>(&p.ws), kBlasWorkspace, "cuBLAS workspace"));
    // RoPE table as the CPU builds it (f5.cpp:529-541): inv = float(1 / 10000^(2j/hd)) in double, angle = float(i) * inv
    // in float, cos/sin of the float angle.
    const int half = d.dim_head / 2;
    std::vector<float2> cs(N * size_t(half));
    for (int j = 0; j < half; ++j) {
        const float inv = float(1.0 / std::pow(10000.0, double(2 * j) / double(d.dim_head)));
        for (size_t i = 0; i < N; ++i) {
            const float a = float(i) * inv;
            cs[i * size_t(half) + size_t(j)] = make_float2(std::cos(a), std::sin(a));
        }
    }
    if (cudaMemcpy(p.cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess) return check_launch("vox_cuda_f5_create");
    if (cudaMemsetAsync(p.h, 0, R * D * 4, user) != cudaSuccess || cudaMemsetAsync(p.ts, 0, D * 4, user) != cudaSuccess)
        return check_launch("vox_cuda_f5_create");
    F5_TRY(blas_check(cublasCreate(&p.blas), "create"));
    F5_TRY(blas_check(cublasSetMathMode(p.blas, d.math == VOX_CUDA_F5_MATH_F32 ? CUBLAS_PEDANTIC_MATH : CUBLAS_DEFAULT_MATH), "math mode"));
    p.compute = d.math == VOX_CUDA_F5_MATH_TF32   ? CUBLAS_COMPUTE_32F_FAST_TF32
                : d.math == VOX_CUDA_F5_MATH_BF16 ? CUBLAS_COMPUTE_32F_FAST_16BF
                                                  : CUBLAS_COMPUTE_32F_PEDANTIC;
    if (cudaStreamCreateWithFlags(&p.cap, cudaStreamNonBlocking) != cudaSuccess) return check_launch("vox_cuda_f5_create");
    // stream and workspace set once, outside the capture (no cuBLAS allocation may happen while capturing)
    F5_TRY(blas_check(cublasSetStream(p.blas, p.cap), "set stream"));
    F5_TRY(blas_check(cublasSetWorkspace(p.blas, p.ws, kBlasWorkspace), "set workspace"));
    // the capture stream starts after the caller's work so far (the table copy and the zeroed inputs)
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return check_launch("vox_cuda_f5_create");
    cudaEventRecord(ev, user);
    cudaStreamWaitEvent(p.cap, ev, 0);
    cudaEventDestroy(ev);
    F5_TRY(record(p, p.cap));  // eager run: algorithm selection and first-use kernel attributes outside the capture
    if (cudaStreamSynchronize(p.cap) != cudaSuccess) return check_launch("vox_cuda_f5_create (eager run)");
    if (cudaStreamBeginCapture(p.cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return check_launch("vox_cuda_f5_create (capture)");
    const int rc = record(p, p.cap);
    const cudaError_t end = cudaStreamEndCapture(p.cap, &p.graph);
    if (rc != VOX_CUDA_OK) return rc;
    if (end != cudaSuccess) return check_launch("vox_cuda_f5_create (end capture)");
    if (cudaGraphInstantiate(&p.exec, p.graph, 0) != cudaSuccess) return check_launch("vox_cuda_f5_create (instantiate)");
    return VOX_CUDA_OK;
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_f5_create(const vox_cuda_f5_desc *desc, void *stream, vox_cuda_f5 **out) {
    VOX_REQUIRE(desc && out, "vox_cuda_f5_create: NULL argument");
    *out = nullptr;
    const vox_cuda_f5_desc &d = *desc;
    VOX_REQUIRE(d.dim > 0 && d.heads > 0 && d.dim_head > 0 && d.dim_head % 2 == 0 && d.ff_mult > 0 && d.depth > 0 && d.out_dim > 0 &&
                    d.batch > 0 && d.frames > 0,
                "vox_cuda_f5_create: bad dimensions");
    VOX_REQUIRE(d.pe_attn_head >= 0 && d.pe_attn_head <= d.heads, "vox_cuda_f5_create: pe_attn_head out of range");
    VOX_REQUIRE(d.math == VOX_CUDA_F5_MATH_F32 || d.math == VOX_CUDA_F5_MATH_TF32 || d.math == VOX_CUDA_F5_MATH_BF16,
                "vox_cuda_f5_create: unknown math mode");
    VOX_REQUIRE(d.blocks && d.norm_out && d.proj_out, "vox_cuda_f5_create: NULL weights");
    for (int i = 0; i < d.depth; ++i) {
        const vox_cuda_f5_block_weights &L = d.blocks[i];
        VOX_REQUIRE(L.ada && L.q && L.k && L.v && L.o && L.ff1 && L.ff2, "vox_cuda_f5_create: NULL block weights");
    }
    const int64_t R = int64_t(d.batch) * d.frames, inner = int64_t(d.heads) * d.dim_head, ff = int64_t(d.ff_mult) * d.dim;
    VOX_REQUIRE(R * std::max<int64_t>(std::max<int64_t>(d.dim, inner), ff) < (int64_t(1) << 31) &&
                    int64_t(d.heads) * d.frames * d.frames < (int64_t(1) << 31) && R * d.heads * (d.dim_head / 2) < (int64_t(1) << 32),
                "vox_cuda_f5_create: problem too large for 32-bit GEMM dimensions");
    F5Plan *p = new F5Plan;
    p->d = d;
    p->blocks.assign(d.blocks, d.blocks + d.depth);
    p->d.blocks = nullptr;
    p->R = R;
    p->inner = inner;
    p->ff = ff;
    const int rc = build(*p, reinterpret_cast<cudaStream_t>(stream));
    if (rc != VOX_CUDA_OK) {
        release(p);
        return rc;
    }
    *out = reinterpret_cast<vox_cuda_f5 *>(p);
    return VOX_CUDA_OK;
}

int vox_cuda_f5_buffers(vox_cuda_f5 *plan, float **h, float **ts, float **out) {
    VOX_REQUIRE(plan, "vox_cuda_f5_buffers: NULL plan");
    F5Plan *p = reinterpret_cast<F5Plan *>(plan);
    if (h) *h = p->h;
    if (ts) *ts = p->ts;
    if (out) *out = p->out;
    return VOX_CUDA_OK;
}

int vox_cuda_f5_run(vox_cuda_f5 *plan, void *stream) {
    VOX_REQUIRE(plan, "vox_cuda_f5_run: NULL plan");
    F5Plan *p = reinterpret_cast<F5Plan *>(plan);
    if (cudaGraphLaunch(p->exec, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return check_launch("vox_cuda_f5_run");
    return VOX_CUDA_OK;
}

void vox_cuda_f5_destroy(vox_cuda_f5 *plan) { release(reinterpret_cast<F5Plan *>(plan)); }

}  // extern "C"
