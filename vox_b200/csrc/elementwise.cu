// Elementwise and broadcast operators: SiLU·mul (SwiGLU), fused gate|up SwiGLU, GELU (erf / tanh), add, mul,
// Snake (three Vox forms), broadcast bias-add and the gated residual add.
//
// All of them stream 16-byte vectors through a grid-stride loop sized to the SM count (kUnroll vectors in flight
// per thread per iteration), with the loads on the read-only path without L1 allocation and the stores .cs, so each
// tensor crosses HBM once. A scalar path serves pointers that are not 16-byte aligned and the tail of n % vector-width
// elements. Per-element parameters (a channel's alpha, a column's bias, a batch's gate) are indexed from the
// vector index with FastDiv, not 64-bit division.
//
// Rounding: where Vox's CPU code (compiled for baseline x86-64, no FMA) rounds after every multiply and add, the
// kernels use __fmul_rn/__fadd_rn so that the only differences from the CPU come from the transcendental
// functions. Vox's own fast_sin polynomial is restated with the same rounded steps, which makes the Kokoro Snake
// bit-exact with the CPU.
//
// Transcendentals are evaluated with fewer instructions than the general-purpose CUDA functions, because the
// bf16 and Snake paths are otherwise bound by instruction issue rather than HBM:
//   sin^2 (HiFT / SnakeBeta): sin^2 has period pi and is even, so theta is reduced by pi with a three-constant
//     Cody-Waite step on FMAs (r in [-pi/2, pi/2]) and sin^2(r) = u * P(u), u = r^2, P a degree-5 polynomial fitted
//     here (weighted least squares on relative error over u in [0, pi^2/4]); max relative error 2.4e-7 in f32,
//     the same as rounding sinf(theta)^2.
//   GELU (erf form): x * Phi(x) with the upper normal tail Q(a) = phi(a) * (b1 t + ... + b5 t^5), t = 1/(1 + p a),
//     from Abramowitz & Stegun 26.2.17 (|error| < 7.5e-8), using the SFU's ex2 and rcp: absolute GELU error below
//     2.5e-7 * |x|, the size of the difference between Vox's two CPU GELUs (std::erf vs nn::gelu_inplace).
//   GELU (tanh form): tanh(z) = 1 - 2 / (1 + e^(2z)) with the SFU's ex2 and rcp (absolute error ~1e-7).
//   SiLU: x / (1 + e^-x) with CUDA's expf and the 2-ulp division (relative error ~3e-7), as kernels.hpp:105.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "sfu.cuh"

namespace voxcuda {
namespace {

constexpr int kThreads = 256;
constexpr int kBlocksPerSm = 8;  // scalar paths
// Vector paths: kUnroll 16-byte vectors per thread per pass and at most kPipeCtasPerSm (one-input ops, software-
// pipelined) or kVecCtasPerSm (two-input ops) CTAs of kThreads per SM. Measured on B200 over 2^25-2^29 elements:
// one-input ops at 2 vectors x 4 CTAs per SM reach 0.96-0.99 of the copy peak against 0.84-0.88 at 4 x 4, and
// two-input ops at 2 x 3 reach 1.00-1.02 against 0.92-0.94 at 4 x 4; more CTAs or deeper passes stream worse.
constexpr int kUnroll = 2;
constexpr int kPipeCtasPerSm = 4;
constexpr int kVecCtasPerSm = 3;

// ------------------------------------------------------------------ scalar math shared by the ops

__device__ __forceinline__ float silu_f(float x) {  // x / (1 + exp(-x)), kernels.hpp:105 (2-ulp division)
    return __fdividef(x, __fadd_rn(1.0f, expf(-x)));
}
// sin^2(theta), two elements per call: Cody-Waite reduction by pi (pi = PI1 + PI2 + PI3, PI1 = float(pi)), then
// u * P(u), u = r^2.
__device__ __forceinline__ float2 sin2_f2(float2 theta) {
    const float2 qq = mul2(theta, bc2(0.31830988618379067f));
    const float2 q = make_float2(rintf(qq.x), rintf(qq.y));
    float2 r = fma2(q, bc2(-3.14159274101257324e+00f), theta);
    r = fma2(q, bc2(8.74227765734758577e-08f), r);
    r = fma2(q, bc2(3.55271367880050093e-15f), r);
    const float2 u = mul2(r, r);
    float2 p = fma2(bc2(-3.60956641998200e-06f), u, bc2(1.39213923830539e-04f));
    p = fma2(p, u, bc2(-3.17209842614830e-03f));
    p = fma2(p, u, bc2(4.44429032504559e-02f));
    p = fma2(p, u, bc2(-3.33332985639572e-01f));
    p = fma2(p, u, bc2(1.0f));
    return mul2(u, p);
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

// Snake: y = x + coef * s^2, s = sin(arg * x). coef is 1/(alpha + 1e-9) (HiFT), inv_b (SnakeBeta) or 1/alpha
// (Kokoro), computed once per channel by the caller. Two elements per call.
template <int KIND>
__device__ __forceinline__ float2 snake_pair(float2 x, float2 arg, float2 coef) {
    if (KIND == VOX_CUDA_SNAKE_KOKORO) {  // kokoro.cpp:237-239, bit-exact with Vox's fast_sin: scalar, unfused roundings
        const float s0 = vox_fast_sin(__fmul_rn(arg.x, x.x)), s1 = vox_fast_sin(__fmul_rn(arg.y, x.y));
        return make_float2(__fadd_rn(x.x, __fmul_rn(coef.x, __fmul_rn(s0, s0))), __fadd_rn(x.y, __fmul_rn(coef.y, __fmul_rn(s1, s1))));
    }
    return add2(x, mul2(coef, sin2_f2(mul2(arg, x))));  // cosyvoice.cpp:243-245 (HiFT), qwen3.cpp:90-91 (SnakeBeta)
}
template <int KIND>
__device__ __forceinline__ float snake_coef(float alpha, float beta) {
    if (KIND == VOX_CUDA_SNAKE_HIFT) return __fdiv_rn(1.0f, __fadd_rn(alpha, 1e-9f));
    if (KIND == VOX_CUDA_SNAKE_BETA) return beta;
    return __fdiv_rn(1.0f, alpha);
}

// ------------------------------------------------------------------ op functors
// Each functor maps W values of the inputs (a, b) starting at element e0 (the first element of a vector, or one
// element on the scalar path, W = 1) to W outputs; W > 1 is processed as W/2 float pairs.

#define VOX_PAIRS(W) for (int k = 0; k < (W); k += 2)
__device__ __forceinline__ float2 pr(const float *v, int k) { return make_float2(v[k], v[k + 1]); }
__device__ __forceinline__ void put(float *y, int k, float2 v) { y[k] = v.x; y[k + 1] = v.y; }

struct OpSiluMul {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *b, float *y, int64_t) const {
#pragma unroll
        for (int k = 0; k < W; ++k) y[k] = __fmul_rn(silu_f(a[k]), b[k]);
    }
};
struct OpAdd {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *b, float *y, int64_t) const {
        if constexpr (W == 1) {
            y[0] = __fadd_rn(a[0], b[0]);
        } else {
#pragma unroll
            VOX_PAIRS(W) put(y, k, add2(pr(a, k), pr(b, k)));
        }
    }
};
struct OpMul {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *b, float *y, int64_t) const {
        if constexpr (W == 1) {
            y[0] = __fmul_rn(a[0], b[0]);
        } else {
#pragma unroll
            VOX_PAIRS(W) put(y, k, mul2(pr(a, k), pr(b, k)));
        }
    }
};
template <int KIND> struct OpGelu {
    template <int W> __device__ __forceinline__ void operator()(const float *a, const float *, float *y, int64_t) const {
        if constexpr (W == 1) {
            const float2 r = KIND == VOX_CUDA_GELU_ERF ? gelu_erf_f2(bc2(a[0])) : gelu_tanh_f2(bc2(a[0]));
            y[0] = r.x;
        } else {
#pragma unroll
            VOX_PAIRS(W) put(y, k, KIND == VOX_CUDA_GELU_ERF ? gelu_erf_f2(pr(a, k)) : gelu_tanh_f2(pr(a, k)));
        }
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
            VOX_PAIRS(W) put(y, k, add2(pr(a, k), make_float2(__ldg(bias + c0 + k), __ldg(bias + c0 + k + 1))));
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
            Vec<DT>::unpack(ld_param(reinterpret_cast<const char *>(gate) + g0 * (DT == VOX_CUDA_F32 ? 4 : 2)), g);
#pragma unroll
            VOX_PAIRS(W) put(y, k, add2(pr(h, k), mul2(pr(g, k), pr(s, k))));
        } else {
            const int64_t gi = (e0 / TD) * D + e0 % D;
            y[0] = __fadd_rn(h[0], __fmul_rn(Vec<DT>::load1(gate, gi), s[0]));
        }
    }
};

// Snake with the channel of element e = (e / inner) % C. On the pipelined path (map_vec_pipe_kernel) each CTA first
// folds every channel's (arg, coef) pair into a shared-memory table when C <= kSnakeTableMax (ntab = C), so a vector
// costs one shared load instead of a global load and a correctly rounded division; elsewhere tab stays NULL and the
// pair is formed per vector. Both give the same bits.
constexpr int64_t kSnakeTableMax = 6144;  // 48 KB of float2: the default dynamic shared-memory limit
template <int KIND> struct OpSnake {
    const float *alpha, *beta;
    FastDiv vrow;  // vector path: vectors per `inner` run (inner % 4 == 0) or vectors per C (inner == 1)
    FastDiv chan;  // C
    int64_t C, inner;
    int time_major;             // inner == 1
    int ntab = 0;               // channels in the per-CTA table (0: no table)
    const float2 *tab = nullptr;  // (arg, coef) per channel in shared memory, set on the device by prepare_op
    template <int W> __device__ __forceinline__ void operator()(const float *x, const float *, float *y, int64_t e0) const {
        if (W > 1 && tab) {
            const uint32_t v = uint32_t(e0 / W);
            if (time_major) {  // W consecutive channels from c0 (a multiple of W): 16-byte aligned table reads
                const float4 *t = reinterpret_cast<const float4 *>(tab + vrow.mod(v) * W);
#pragma unroll
                VOX_PAIRS(W) {
                    const float4 p = t[k / 2];
                    put(y, k, snake_pair<KIND>(pr(x, k), make_float2(p.x, p.z), make_float2(p.y, p.w)));
                }
            } else {
                const float2 p = tab[chan.mod(vrow.div(v))];
                const float2 arg = bc2(p.x), cf = bc2(p.y);
#pragma unroll
                VOX_PAIRS(W) put(y, k, snake_pair<KIND>(pr(x, k), arg, cf));
            }
        } else if (W > 1) {
            const uint32_t v = uint32_t(e0 / W);
            if (time_major) {
                const int64_t c0 = int64_t(vrow.mod(v)) * W;
#pragma unroll
                VOX_PAIRS(W) {
                    const float a0 = __ldg(alpha + c0 + k), a1 = __ldg(alpha + c0 + k + 1);
                    const float b0 = KIND == VOX_CUDA_SNAKE_BETA ? __ldg(beta + c0 + k) : 0.f;
                    const float b1 = KIND == VOX_CUDA_SNAKE_BETA ? __ldg(beta + c0 + k + 1) : 0.f;
                    put(y, k, snake_pair<KIND>(pr(x, k), make_float2(a0, a1), make_float2(snake_coef<KIND>(a0, b0), snake_coef<KIND>(a1, b1))));
                }
            } else {
                const uint32_t c = chan.mod(vrow.div(v));
                const float al = __ldg(alpha + c);
                const float2 arg = bc2(al), cf = bc2(snake_coef<KIND>(al, KIND == VOX_CUDA_SNAKE_BETA ? __ldg(beta + c) : 0.f));
#pragma unroll
                VOX_PAIRS(W) put(y, k, snake_pair<KIND>(pr(x, k), arg, cf));
            }
        } else {
            const int64_t c = (e0 / inner) % C;
            const float2 r = snake_pair<KIND>(bc2(x[0]), bc2(alpha[c]), bc2(snake_coef<KIND>(alpha[c], KIND == VOX_CUDA_SNAKE_BETA ? beta[c] : 0.f)));
            y[0] = r.x;
        }
    }
};

// Per-CTA shared tables of the pipelined path: a no-op for every functor but Snake.
template <class F> __device__ __forceinline__ void prepare_op(F &, float2 *) {}
template <int KIND> __device__ __forceinline__ void prepare_op(OpSnake<KIND> &f, float2 *tab) {
    if (f.ntab == 0) return;
    for (int c = threadIdx.x; c < f.ntab; c += blockDim.x) {
        const float al = __ldg(f.alpha + c);
        tab[c] = make_float2(al, snake_coef<KIND>(al, KIND == VOX_CUDA_SNAKE_BETA ? __ldg(f.beta + c) : 0.f));
    }
    __syncthreads();
    f.tab = tab;
}
template <class F> size_t op_table_bytes(const F &) { return 0; }
template <int KIND> size_t op_table_bytes(const OpSnake<KIND> &f) { return size_t(f.ntab) * sizeof(float2); }

// ------------------------------------------------------------------ kernels

// Vector paths. A launch covers at most kMaxLaunchVecs 16-byte vectors, so vector indices are 32-bit (no index
// formed below exceeds nvec by more than 2 * kUnroll grid strides); the host splits longer tensors into launches
// whose pointers start at the launch's first element and passes that element's index as `base`, which the functors
// see added to e0. The n % W tail (last launch only) is mapped by block 0.
constexpr int64_t kMaxLaunchVecs = int64_t(1) << 30;

// Two-input ops: kUnroll vectors of each input in flight per thread per pass (the last pass predicated).
template <int DT, int NIN, class F>
__global__ void __launch_bounds__(kThreads, kVecCtasPerSm) map_vec_kernel(const void *a, const void *b, void *y, int64_t n, int64_t base, F f) {
    pdl_enter();
    using V = Vec<DT>;
    constexpr int W = V::N;
    const uint32_t nvec = uint32_t(n / W);
    const uint32_t stride = gridDim.x * blockDim.x;
    const uint4 *pa = reinterpret_cast<const uint4 *>(a);
    const uint4 *pb = reinterpret_cast<const uint4 *>(b);
    uint4 *py = reinterpret_cast<uint4 *>(y);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += kUnroll * stride) {
        uint4 ra[kUnroll], rb[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t j = i + u * stride;
            if (j < nvec) {
                ra[u] = ld_stream(pa + j);
                if (NIN == 2) rb[u] = ld_stream(pb + j);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t j = i + u * stride;
            if (j < nvec) {
                float fa[W], fb[W], fy[W];
                V::unpack(ra[u], fa);
                if (NIN == 2) V::unpack(rb[u], fb);
                f.template operator()<W>(fa, fb, fy, base + int64_t(j) * W);
                st_stream(py + j, V::pack(fy));
            }
        }
    }
    const int64_t tail = n - int64_t(nvec) * W;
    if (blockIdx.x == 0 && int64_t(threadIdx.x) < tail) {
        const int64_t e = int64_t(nvec) * W + threadIdx.x;
        float fa[1], fb[1] = {0.f}, fy[1];
        fa[0] = V::load1(a, e);
        if (NIN == 2) fb[0] = V::load1(b, e);
        f.template operator()<1>(fa, fb, fy, base + e);
        V::store1(y, e, fy[0]);
    }
}

// One-input ops (GELU, Snake, bias-add), software-pipelined: the loads of a thread's next pass are issued before the
// current pass is computed, so the arithmetic of one pass overlaps the memory latency of the next (these ops carry
// the most instructions per byte of the library).
template <int DT, class F>
__global__ void __launch_bounds__(kThreads, kPipeCtasPerSm) map_vec_pipe_kernel(const void *a, void *y, int64_t n, int64_t base, F f) {
    pdl_enter();
    extern __shared__ float2 map_op_table[];
    prepare_op(f, map_op_table);
    using V = Vec<DT>;
    constexpr int W = V::N;
    const uint32_t nvec = uint32_t(n / W);
    const uint32_t stride = gridDim.x * blockDim.x;
    const uint4 *pa = reinterpret_cast<const uint4 *>(a);
    uint4 *py = reinterpret_cast<uint4 *>(y);
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    uint4 cur[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
        if (i + u * stride < nvec) cur[u] = ld_stream(pa + i + u * stride);
    for (; i < nvec; i += kUnroll * stride) {
        const uint32_t inext = i + kUnroll * stride;
        uint4 nxt[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
            if (inext + u * stride < nvec) nxt[u] = ld_stream(pa + inext + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t j = i + u * stride;
            if (j < nvec) {
                float fa[W], fy[W];
                V::unpack(cur[u], fa);
                f.template operator()<W>(fa, fa, fy, base + int64_t(j) * W);
                st_stream(py + j, V::pack(fy));
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) cur[u] = nxt[u];
    }
    const int64_t tail = n - int64_t(nvec) * W;
    if (blockIdx.x == 0 && int64_t(threadIdx.x) < tail) {
        const int64_t e = int64_t(nvec) * W + threadIdx.x;
        float fa[1], fy[1];
        fa[0] = V::load1(a, e);
        f.template operator()<1>(fa, fa, fy, base + e);
        V::store1(y, e, fy[0]);
    }
}

// Scalar path for unaligned pointers or shapes the vector path cannot index.
template <int DT, int NIN, class F>
__global__ void __launch_bounds__(kThreads) map_scalar_kernel(const void *a, const void *b, void *y, int64_t n, F f) {
    pdl_enter();
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

// The software-pipelined one-input path; VOX_CUDA_MAP_PIPE=0 selects the plain vector path (for comparisons).
bool map_pipe_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("VOX_CUDA_MAP_PIPE");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <int DT, int NIN, class F>
int launch_map(const void *a, const void *b, void *y, int64_t n, F f, bool vec_ok, cudaStream_t st, const char *name) {
    if (n == 0) return VOX_CUDA_OK;
    constexpr int W = Vec<DT>::N;
    constexpr int64_t esize = DT == VOX_CUDA_F32 ? 4 : 2;
    // the functors index per-vector parameters with 32-bit vector indices
    vec_ok = vec_ok && aligned16(a) && aligned16(y) && (NIN == 1 || aligned16(b)) && n / W < (int64_t(1) << 32);
    if (!vec_ok) {
        const int g = grid_for(n, kThreads, kBlocksPerSm);
        launch_k(map_scalar_kernel<DT, NIN, F>, g, kThreads, 0, st, a, b, y, n, f);
        return check_launch(name);
    }
    const bool pipe = NIN == 1 && map_pipe_enabled();
    const void *kern = pipe ? (const void *)map_vec_pipe_kernel<DT, F> : (const void *)map_vec_kernel<DT, NIN, F>;
    const size_t smem = pipe ? op_table_bytes(f) : 0;
    const int cap = (pipe ? kPipeCtasPerSm : kVecCtasPerSm) * sm_count();
    const int resident = std::min(resident_blocks(kern, kThreads, smem), cap);
    const int64_t nvec = n / W;
    for (int64_t v0 = 0; v0 == 0 || v0 < nvec; v0 += kMaxLaunchVecs) {
        const int64_t nv = std::min(kMaxLaunchVecs, nvec - v0);
        const int64_t e0 = v0 * W, ne = v0 + nv == nvec ? n - e0 : nv * W;  // the last launch takes the tail
        const char *ca = static_cast<const char *>(a) + e0 * esize;
        const char *cb = NIN == 2 ? static_cast<const char *>(b) + e0 * esize : nullptr;
        char *cy = static_cast<char *>(y) + e0 * esize;
        const int g = balanced_grid(std::max<int64_t>(nv, 1), int64_t(kThreads) * kUnroll, resident);
        if (pipe) launch_k(map_vec_pipe_kernel<DT, F>, g, kThreads, smem, st, (const void *)ca, (void *)cy, ne, e0, f);
        else launch_k(map_vec_kernel<DT, NIN, F>, g, kThreads, 0, st, (const void *)ca, (const void *)cb, (void *)cy, ne, e0, f);
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
    pdl_enter();
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
    pdl_enter();
    using V = Vec<DT>;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < m * I; i += stride) {
        const int64_t r = i / I, e = i - r * I;
        V::store1(h, i, __fmul_rn(silu_f(V::load1(gu, r * 2 * I + e)), V::load1(gu, r * 2 * I + I + e)));
    }
}

__global__ void snake_params_kernel(const float *alpha, const float *beta, float *a, float *inv_b, int64_t C) {
    pdl_enter();
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
    const int ntab = vec_ok && C <= kSnakeTableMax ? int(C) : 0;
    auto run = [&](auto op) {
        op.ntab = ntab;
        return dispatch_map<1>(VOX_CUDA_F32, x, nullptr, y, n, op, vec_ok, stream, "vox_cuda_snake");
    };
    switch (kind) {
        case VOX_CUDA_SNAKE_HIFT: return run(OpSnake<VOX_CUDA_SNAKE_HIFT>{alpha, beta, vrow, chan, C, inner, tm});
        case VOX_CUDA_SNAKE_BETA: return run(OpSnake<VOX_CUDA_SNAKE_BETA>{alpha, beta, vrow, chan, C, inner, tm});
        default: return run(OpSnake<VOX_CUDA_SNAKE_KOKORO>{alpha, beta, vrow, chan, C, inner, tm});
    }
}

int vox_cuda_snake_beta_params(const float *alpha, const float *beta, float *a, float *inv_b, int64_t C, void *stream) {
    VOX_REQUIRE(C >= 0 && (C == 0 || (alpha && beta && a && inv_b)), "vox_cuda_snake_beta_params: bad arguments");
    if (C == 0) return VOX_CUDA_OK;
    launch_k(snake_params_kernel, int((C + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream), alpha, beta, a, inv_b, C);
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
        if (dtype == VOX_CUDA_F32) launch_k(swiglu_fused_kernel<VOX_CUDA_F32>, g, kThreads, 0, st, gu, h, m, I, FastDiv(uint32_t(I / W)));
        else launch_k(swiglu_fused_kernel<VOX_CUDA_BF16>, g, kThreads, 0, st, gu, h, m, I, FastDiv(uint32_t(I / W)));
    } else {
        const int g = grid_for(m * I, kThreads, kBlocksPerSm);
        if (dtype == VOX_CUDA_F32) launch_k(swiglu_fused_scalar<VOX_CUDA_F32>, g, kThreads, 0, st, gu, h, m, I);
        else launch_k(swiglu_fused_scalar<VOX_CUDA_BF16>, g, kThreads, 0, st, gu, h, m, I);
    }
    return check_launch("vox_cuda_swiglu_fused");
}

}  // extern "C"
