// Elementwise and broadcast operators: SiLU·mul (SwiGLU), fused gate|up SwiGLU, GELU (erf / tanh), add, mul,
// Snake (three Vox forms), broadcast bias-add and the gated residual add.
//
// All of them stream 16-byte vectors through a grid-stride loop sized to the SM count (U vectors in flight per
// thread per iteration), with the loads marked L1::no_allocate + L2::evict_first and the stores .cs, so each tensor
// crosses HBM once. A scalar path serves pointers that are not 16-byte aligned and the tail of n % vector-width
// elements. Per-element parameters (a channel's alpha, a column's bias, a batch's gate) are indexed from the
// vector index with FastDiv, not 64-bit division.
//
// Rounding: where Vox's CPU code (compiled for baseline x86-64, no FMA) rounds after every multiply and add, the
// kernels use __fmul_rn/__fadd_rn so that the only differences from the CPU come from the transcendental
// functions (expf/erff/tanhf/sinf of CUDA vs glibc). Vox's own fast_sin polynomial is restated with the same
// rounded steps, which makes the Kokoro Snake bit-exact with the CPU.
#include "common.cuh"

namespace voxcuda {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kBlocksPerSm = 8;

// ------------------------------------------------------------------ scalar math shared by the ops

__device__ __forceinline__ float silu_f(float x) {  // x / (1 + exp(-x)), kernels.hpp:105
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}
__device__ __forceinline__ float gelu_erf_f(float x) {  // 0.5 x (1 + erf(x / sqrt2)), kernels.hpp:106
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752440f))));
}
__device__ __forceinline__ float gelu_tanh_f(float x) {  // f5.cpp:93-96
    const float k = 0.7978845608028654f;
    const float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(__fmul_rn(k, __fadd_rn(x, x3)))));
}

// Vox's fast_sin (nn.hpp:26-40): reduction by pi in three parts, odd polynomial of degree 11, sign from the
// parity of the quotient. Every step rounded separately, as the CPU build computes it.
__device__ __forceinline__ float vox_fast_sin(float x) {
    const float q = rintf(__fmul_rn(x, 0.31830988618379067f));
    float r = __fsub_rn(x, __fmul_rn(q, 3.140625f));
    r = __fsub_rn(r, __fmul_rn(q, 9.67502593994140625e-4f));
    r = __fsub_rn(r, __fmul_rn(q, 1.509957990978376432e-7f));
    const float r2 = __fmul_rn(r, r);
    float p = -2.39e-8f;
    p = __fadd_rn(__fmul_rn(p, r2), 2.7526e-6f);
    p = __fsub_rn(__fmul_rn(p, r2), 1.98409e-4f);
    p = __fadd_rn(__fmul_rn(p, r2), 8.3333315e-3f);
    p = __fsub_rn(__fmul_rn(p, r2), 1.6666666e-1f);
    const float s = __fadd_rn(r, __fmul_rn(__fmul_rn(r, r2), p));
    const int qi = int(q);
    return (qi & 1) ? -s : s;
}

// One Snake element: y = x + coef * s^2, s = sin(arg * x), in the rounding order of the CPU forms.
template <int KIND>
__device__ __forceinline__ float snake_elem(float x, float al, float be) {
    if (KIND == VOX_CUDA_SNAKE_HIFT) {  // cosyvoice.cpp:243-245
        const float s = sinf(__fmul_rn(al, x));
        return __fadd_rn(x, __fmul_rn(__fdiv_rn(1.0f, __fadd_rn(al, 1e-9f)), __fmul_rn(s, s)));
    } else if (KIND == VOX_CUDA_SNAKE_BETA) {  // qwen3.cpp:90-91: v + inv_b * sn * sn, sn = sin(v * a)
        const float s = sinf(__fmul_rn(x, al));
        return __fadd_rn(x, __fmul_rn(__fmul_rn(be, s), s));
    } else {  // kokoro.cpp:237-239
        const float s = vox_fast_sin(__fmul_rn(al, x));
        return __fadd_rn(x, __fmul_rn(__fdiv_rn(1.0f, al), __fmul_rn(s, s)));
    }
}

// ------------------------------------------------------------------ op functors
// Each functor maps W values of the inputs (a, b) starting at element e0 (the first element of a vector, or one
// element on the scalar path) to W outputs.

struct OpSiluMul {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *b, float *y, int64_t) const {
#pragma unroll
        for (int k = 0; k < W; ++k) y[k] = __fmul_rn(silu_f(a[k]), b[k]);
    }
};
struct OpAdd {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *b, float *y, int64_t) const {
#pragma unroll
        for (int k = 0; k < W; ++k) y[k] = __fadd_rn(a[k], b[k]);
    }
};
struct OpMul {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *b, float *y, int64_t) const {
#pragma unroll
        for (int k = 0; k < W; ++k) y[k] = __fmul_rn(a[k], b[k]);
    }
};
template <int KIND> struct OpGelu {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *, float *y, int64_t) const {
#pragma unroll
        for (int k = 0; k < W; ++k) y[k] = KIND == VOX_CUDA_GELU_ERF ? gelu_erf_f(a[k]) : gelu_tanh_f(a[k]);
    }
};

// y[r][o] = y[r][o] + bias[o]: element e has column e % D.
struct OpBias {
    const float *bias;
    FastDiv vpr;  // vectors per row (vector path) or D (scalar path)
    int64_t D;
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *, float *y, int64_t e0) const {
        if (W > 1) {
            const uint32_t v = uint32_t(e0 / W);
            const int64_t c0 = int64_t(vpr.mod(v)) * W;
#pragma unroll
            for (int k = 0; k < W; ++k) y[k] = __fadd_rn(a[k], __ldg(bias + c0 + k));
        } else {
            y[0] = __fadd_rn(a[0], __ldg(bias + e0 % D));
        }
    }
};

// h = h + gate[b][d] * src: element e of [B][T][D] has batch e / (T*D) and column e % D.
template <int DT> struct OpGated {
    const void *gate;
    FastDiv vpr;    // vectors per row
    FastDiv vpb;    // vectors per batch
    int64_t D, TD;  // scalar path
    template <int W> __device__ __forceinline__ void operator()(const float *h, const float *s, float *y, int64_t e0) const {
        if (W > 1) {
            const uint32_t v = uint32_t(e0 / W);
            const int64_t g0 = int64_t(vpb.div(v)) * D + int64_t(vpr.mod(v)) * W;
            float g[W];
            Vec<DT>::unpack(ld_param(reinterpret_cast<const char *>(gate) + g0 * dtype_size_dev()), g);
#pragma unroll
            for (int k = 0; k < W; ++k) y[k] = __fadd_rn(h[k], __fmul_rn(g[k], s[k]));
        } else {
            const int64_t gi = (e0 / TD) * D + e0 % D;
            y[0] = __fadd_rn(h[0], __fmul_rn(Vec<DT>::load1(gate, gi), s[0]));
        }
    }
    __device__ __forceinline__ static int64_t dtype_size_dev() { return DT == VOX_CUDA_F32 ? 4 : 2; }
};

// Snake with the channel of element e = (e / inner) % C.
template <int KIND> struct OpSnake {
    const float *alpha, *beta;
    FastDiv vrow;  // vector path: vectors per `inner` run (inner % 4 == 0) or vectors per C (inner == 1)
    FastDiv chan;  // C
    int64_t C, inner;
    int time_major;  // inner == 1
    template <int W> __device__ __forceinline__ void operator()(const float *x, const float *, float *y, int64_t e0) const {
        if (W > 1) {
            const uint32_t v = uint32_t(e0 / W);
            if (time_major) {
                const int64_t c0 = int64_t(vrow.mod(v)) * W;
#pragma unroll
                for (int k = 0; k < W; ++k)
                    y[k] = snake_elem<KIND>(x[k], __ldg(alpha + c0 + k), KIND == VOX_CUDA_SNAKE_BETA ? __ldg(beta + c0 + k) : 0.f);
            } else {
                const uint32_t c = chan.mod(vrow.div(v));
                const float al = __ldg(alpha + c), be = KIND == VOX_CUDA_SNAKE_BETA ? __ldg(beta + c) : 0.f;
#pragma unroll
                for (int k = 0; k < W; ++k) y[k] = snake_elem<KIND>(x[k], al, be);
            }
        } else {
            const int64_t c = (e0 / inner) % C;
            y[0] = snake_elem<KIND>(x[0], alpha[c], KIND == VOX_CUDA_SNAKE_BETA ? beta[c] : 0.f);
        }
    }
};

// ------------------------------------------------------------------ kernels

// Vector path: n / W 16-byte vectors, U of them in flight per thread, then the n % W tail by block 0.
template <int DT, int NIN, class F>
__global__ void __launch_bounds__(kThreads) map_vec_kernel(const void *a, const void *b, void *y, int64_t n, F f) {
    using V = Vec<DT>;
    constexpr int W = V::N;
    const int64_t nvec = n / W;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint4 *pa = reinterpret_cast<const uint4 *>(a);
    const uint4 *pb = reinterpret_cast<const uint4 *>(b);
    uint4 *py = reinterpret_cast<uint4 *>(y);
    for (; i + (kUnroll - 1) * stride < nvec; i += kUnroll * stride) {
        uint4 ra[kUnroll], rb[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            ra[u] = ld_stream(pa + i + u * stride);
            if (NIN == 2) rb[u] = ld_stream(pb + i + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            float fa[W], fb[W], fy[W];
            V::unpack(ra[u], fa);
            if (NIN == 2) V::unpack(rb[u], fb);
            f.template operator()<W>(fa, fb, fy, (i + u * stride) * W);
            st_stream(py + i + u * stride, V::pack(fy));
        }
    }
    for (; i < nvec; i += stride) {
        float fa[W], fb[W], fy[W];
        V::unpack(ld_stream(pa + i), fa);
        if (NIN == 2) V::unpack(ld_stream(pb + i), fb);
        f.template operator()<W>(fa, fb, fy, i * W);
        st_stream(py + i, V::pack(fy));
    }
    const int64_t tail = n - nvec * W;
    if (blockIdx.x == 0 && int64_t(threadIdx.x) < tail) {
        const int64_t e = nvec * W + threadIdx.x;
        float fa[1], fb[1] = {0.f}, fy[1];
        fa[0] = V::load1(a, e);
        if (NIN == 2) fb[0] = V::load1(b, e);
        f.template operator()<1>(fa, fb, fy, e);
        V::store1(y, e, fy[0]);
    }
}

// Scalar path for unaligned pointers or shapes the vector path cannot index.
template <int DT, int NIN, class F>
__global__ void __launch_bounds__(kThreads) map_scalar_kernel(const void *a, const void *b, void *y, int64_t n, F f) {
    using V = Vec<DT>;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += stride) {
        float fa[1], fb[1] = {0.f}, fy[1];
        fa[0] = V::load1(a, e);
        if (NIN == 2) fb[0] = V::load1(b, e);
        f.template operator()<1>(fa, fb, fy, e);
        V::store1(y, e, fy[0]);
    }
}

template <int DT, int NIN, class F>
int launch_map(const void *a, const void *b, void *y, int64_t n, F f, bool vec_ok, cudaStream_t st, const char *name) {
    if (n == 0) return VOX_CUDA_OK;
    constexpr int W = Vec<DT>::N;
    vec_ok = vec_ok && aligned16(a) && aligned16(y) && (NIN == 1 || aligned16(b)) && n / W < (int64_t(1) << 32);
    if (vec_ok) {
        const int g = grid_for((n / W + kUnroll - 1) / kUnroll, kThreads, kBlocksPerSm);
        map_vec_kernel<DT, NIN, F><<<g, kThreads, 0, st>>>(a, b, y, n, f);
    } else {
        const int g = grid_for(n, kThreads, kBlocksPerSm);
        map_scalar_kernel<DT, NIN, F><<<g, kThreads, 0, st>>>(a, b, y, n, f);
    }
    return check_launch(name);
}

template <int NIN, class F>
int dispatch_map(int dtype, const void *a, const void *b, void *y, int64_t n, F f, bool vec_ok, void *stream, const char *name) {
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == VOX_CUDA_F32) return launch_map<VOX_CUDA_F32, NIN>(a, b, y, n, f, vec_ok, st, name);
    return launch_map<VOX_CUDA_BF16, NIN>(a, b, y, n, f, vec_ok, st, name);
}

// ------------------------------------------------------------------ fused gate|up SwiGLU (swiglu.comp layout)

// gu [m][2I] -> h [m][I]. One thread per 16-byte output vector; row index by FastDiv on the vector index.
template <int DT>
__global__ void __launch_bounds__(kThreads) swiglu_fused_kernel(const void *gu, void *h, int64_t m, int64_t I, FastDiv vpr) {
    using V = Vec<DT>;
    constexpr int W = V::N;
    const int64_t nvec = m * I / W;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t rowbytes = 2 * I * (DT == VOX_CUDA_F32 ? 4 : 2);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
        const uint32_t r = vpr.div(uint32_t(i));
        const int64_t c = int64_t(uint32_t(i) - r * vpr.d);
        const char *row = reinterpret_cast<const char *>(gu) + int64_t(r) * rowbytes;
        const uint4 ga = ld_stream(row + c * 16), ua = ld_stream(row + rowbytes / 2 + c * 16);
        float fg[W], fu[W], fy[W];
        V::unpack(ga, fg);
        V::unpack(ua, fu);
#pragma unroll
        for (int k = 0; k < W; ++k) fy[k] = __fmul_rn(silu_f(fg[k]), fu[k]);
        st_stream(reinterpret_cast<uint4 *>(h) + i, V::pack(fy));
    }
}

template <int DT>
__global__ void __launch_bounds__(kThreads) swiglu_fused_scalar(const void *gu, void *h, int64_t m, int64_t I) {
    using V = Vec<DT>;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < m * I; i += stride) {
        const int64_t r = i / I, e = i - r * I;
        V::store1(h, i, __fmul_rn(silu_f(V::load1(gu, r * 2 * I + e)), V::load1(gu, r * 2 * I + I + e)));
    }
}

__global__ void snake_params_kernel(const float *alpha, const float *beta, float *a, float *inv_b, int64_t C) {
    const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (c < C) {
        a[c] = expf(alpha[c]);
        inv_b[c] = __fdiv_rn(1.0f, __fadd_rn(expf(beta[c]), 1e-9f));
    }
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_silu_mul(const void *g, const void *u, void *h, int64_t n, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_silu_mul: dtype must be F32 or BF16");
    VOX_REQUIRE(n >= 0 && (n == 0 || (g && u && h)), "vox_cuda_silu_mul: bad pointers or size");
    return dispatch_map<2>(dtype, g, u, h, n, OpSiluMul{}, true, stream, "vox_cuda_silu_mul");
}

int vox_cuda_add(const void *a, const void *b, void *y, int64_t n, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_add: dtype must be F32 or BF16");
    VOX_REQUIRE(n >= 0 && (n == 0 || (a && b && y)), "vox_cuda_add: bad pointers or size");
    return dispatch_map<2>(dtype, a, b, y, n, OpAdd{}, true, stream, "vox_cuda_add");
}

int vox_cuda_mul(const void *a, const void *b, void *y, int64_t n, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_mul: dtype must be F32 or BF16");
    VOX_REQUIRE(n >= 0 && (n == 0 || (a && b && y)), "vox_cuda_mul: bad pointers or size");
    return dispatch_map<2>(dtype, a, b, y, n, OpMul{}, true, stream, "vox_cuda_mul");
}

int vox_cuda_gelu(const void *x, void *y, int64_t n, int kind, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_gelu: dtype must be F32 or BF16");
    VOX_REQUIRE(kind == VOX_CUDA_GELU_ERF || kind == VOX_CUDA_GELU_TANH, "vox_cuda_gelu: unknown kind");
    VOX_REQUIRE(n >= 0 && (n == 0 || (x && y)), "vox_cuda_gelu: bad pointers or size");
    if (kind == VOX_CUDA_GELU_ERF) return dispatch_map<1>(dtype, x, nullptr, y, n, OpGelu<VOX_CUDA_GELU_ERF>{}, true, stream, "vox_cuda_gelu");
    return dispatch_map<1>(dtype, x, nullptr, y, n, OpGelu<VOX_CUDA_GELU_TANH>{}, true, stream, "vox_cuda_gelu");
}

int vox_cuda_bias_add(void *y, const float *b, int64_t rows, int64_t D, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_bias_add: dtype must be F32 or BF16");
    VOX_REQUIRE(rows >= 0 && D > 0, "vox_cuda_bias_add: bad shape");
    VOX_REQUIRE(rows == 0 || (y && b), "vox_cuda_bias_add: NULL pointer");
    const int W = dtype == VOX_CUDA_F32 ? 4 : 8;
    const bool vec_ok = D % W == 0 && D / W < (int64_t(1) << 32);
    OpBias op{b, FastDiv(vec_ok ? uint32_t(D / W) : 1u), D};
    return dispatch_map<1>(dtype, y, nullptr, y, rows * D, op, vec_ok, stream, "vox_cuda_bias_add");
}

int vox_cuda_gated_add(void *h, const void *gate, const void *src, int64_t B, int64_t T, int64_t D, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_gated_add: dtype must be F32 or BF16");
    VOX_REQUIRE(B >= 0 && T >= 0 && D > 0, "vox_cuda_gated_add: bad shape");
    const int64_t n = B * T * D;
    VOX_REQUIRE(n == 0 || (h && gate && src), "vox_cuda_gated_add: NULL pointer");
    if (n == 0) return VOX_CUDA_OK;
    const int W = dtype == VOX_CUDA_F32 ? 4 : 8;
    const bool vec_ok = D % W == 0 && aligned16(gate) && (T * D) / W < (int64_t(1) << 32);
    if (dtype == VOX_CUDA_F32) {
        OpGated<VOX_CUDA_F32> op{gate, FastDiv(vec_ok ? uint32_t(D / W) : 1u), FastDiv(vec_ok ? uint32_t(T * D / W) : 1u), D, T * D};
        return dispatch_map<2>(dtype, h, src, h, n, op, vec_ok, stream, "vox_cuda_gated_add");
    }
    OpGated<VOX_CUDA_BF16> op{gate, FastDiv(vec_ok ? uint32_t(D / W) : 1u), FastDiv(vec_ok ? uint32_t(T * D / W) : 1u), D, T * D};
    return dispatch_map<2>(dtype, h, src, h, n, op, vec_ok, stream, "vox_cuda_gated_add");
}

int vox_cuda_snake(const float *x, const float *alpha, const float *beta, float *y, int64_t n, int64_t C, int64_t inner, int kind,
                   void *stream) {
    VOX_REQUIRE(kind == VOX_CUDA_SNAKE_HIFT || kind == VOX_CUDA_SNAKE_BETA || kind == VOX_CUDA_SNAKE_KOKORO,
                "vox_cuda_snake: unknown kind");
    VOX_REQUIRE(n >= 0 && C > 0 && inner > 0, "vox_cuda_snake: bad shape");
    VOX_REQUIRE(n == 0 || (x && y && alpha), "vox_cuda_snake: NULL pointer");
    VOX_REQUIRE(kind != VOX_CUDA_SNAKE_BETA || beta, "vox_cuda_snake: BETA needs beta (inv_b)");
    const bool time_major = inner == 1;
    bool vec_ok = time_major ? (C % 4 == 0) : (inner % 4 == 0);
    vec_ok = vec_ok && (time_major ? C / 4 : inner / 4) < (int64_t(1) << 32) && C < (int64_t(1) << 32);
    FastDiv vrow(vec_ok ? uint32_t(time_major ? C / 4 : inner / 4) : 1u), chan(uint32_t(C < (int64_t(1) << 32) ? C : 1));
    const int tm = time_major ? 1 : 0;
    switch (kind) {
        case VOX_CUDA_SNAKE_HIFT:
            return dispatch_map<1>(VOX_CUDA_F32, x, nullptr, y, n, OpSnake<VOX_CUDA_SNAKE_HIFT>{alpha, beta, vrow, chan, C, inner, tm},
                                   vec_ok, stream, "vox_cuda_snake");
        case VOX_CUDA_SNAKE_BETA:
            return dispatch_map<1>(VOX_CUDA_F32, x, nullptr, y, n, OpSnake<VOX_CUDA_SNAKE_BETA>{alpha, beta, vrow, chan, C, inner, tm},
                                   vec_ok, stream, "vox_cuda_snake");
        default:
            return dispatch_map<1>(VOX_CUDA_F32, x, nullptr, y, n,
                                   OpSnake<VOX_CUDA_SNAKE_KOKORO>{alpha, beta, vrow, chan, C, inner, tm}, vec_ok, stream,
                                   "vox_cuda_snake");
    }
}

int vox_cuda_snake_beta_params(const float *alpha, const float *beta, float *a, float *inv_b, int64_t C, void *stream) {
    VOX_REQUIRE(C >= 0 && (C == 0 || (alpha && beta && a && inv_b)), "vox_cuda_snake_beta_params: bad arguments");
    if (C == 0) return VOX_CUDA_OK;
    snake_params_kernel<<<int((C + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(alpha, beta, a, inv_b, C);
    return check_launch("vox_cuda_snake_beta_params");
}

int vox_cuda_swiglu_fused(const void *gu, void *h, int64_t m, int64_t I, int dtype, void *stream) {
    VOX_REQUIRE(is_act_dtype(dtype), "vox_cuda_swiglu_fused: dtype must be F32 or BF16");
    VOX_REQUIRE(m >= 0 && I > 0, "vox_cuda_swiglu_fused: bad shape");
    VOX_REQUIRE(m == 0 || (gu && h), "vox_cuda_swiglu_fused: NULL pointer");
    if (m == 0) return VOX_CUDA_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int W = dtype == VOX_CUDA_F32 ? 4 : 8;
    const bool vec_ok = I % W == 0 && aligned16(gu) && aligned16(h) && m * I / W < (int64_t(1) << 32);
    if (vec_ok) {
        const int g = grid_for(m * I / W, kThreads, kBlocksPerSm);
        if (dtype == VOX_CUDA_F32) swiglu_fused_kernel<VOX_CUDA_F32><<<g, kThreads, 0, st>>>(gu, h, m, I, FastDiv(uint32_t(I / W)));
        else swiglu_fused_kernel<VOX_CUDA_BF16><<<g, kThreads, 0, st>>>(gu, h, m, I, FastDiv(uint32_t(I / W)));
    } else {
        const int g = grid_for(m * I, kThreads, kBlocksPerSm);
        if (dtype == VOX_CUDA_F32) swiglu_fused_scalar<VOX_CUDA_F32><<<g, kThreads, 0, st>>>(gu, h, m, I);
        else swiglu_fused_scalar<VOX_CUDA_BF16><<<g, kThreads, 0, st>>>(gu, h, m, I);
    }
    return check_launch("vox_cuda_swiglu_fused");
}

}  // extern "C"
