// The per-token elementwise steps of a transformer layer between its fused QKV projection and its attention:
// the RoPE cos/sin table (vox_cuda_rope_table) and one fused pass that splits the projection, applies the optional
// q/k head RMSNorm and the rotate-half RoPE, and writes q and the token's K and V cache rows (vox_cuda_qkv_rope).
//
// Vox runs these as three GPU dispatches per layer (shaders/qkvsplit.comp, then shaders/qkrope.comp once over q and
// once over the K cache rows, in place) or, on the CPU, as per-head vox::rmsnorm + vox::rope_apply calls per token
// (kernels.cpp:797-803) followed by appends to the caches. Here every projection element is read once and written
// once: one warp per head of one token (q heads, then k heads, then v heads), the head held in registers, the
// rotation partner (element e + hd/2) fetched with one shuffle from lane ^ 16.
//
// Arithmetic follows the CPU: the head norm is w * (x * inv) with inv = 1 / sqrt(ss / hd + eps) (kernels.cpp:707-712;
// ss summed by a warp butterfly instead of sequentially, a difference of ~1e-7 relative), and the rotation is
// a*c - b*s, b*c + a*s with every product rounded separately (kernels.cpp:753-754), so with the table of the same
// cos/sin values and no head norm the result is bit-identical to the CPU. The table itself is computed on the
// device with CUDA's sincosf of f = inv_freq[p] * float(pos) (kernels.cpp:745-747 uses libm's cosf/sinf of the same
// f; both are within 2 ulp of the true values).
#include <math.h>

#include "common.cuh"

namespace voxcuda {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct QkvRopeArgs {
    const float *qkv;           // [m][stride], stride = qd + 2 kd
    const float *qn, *kn;       // head-norm weights [hd] or NULL
    const float *cs;            // [m][hd/2][2]
    float *q, *kc, *vc;         // [m][qd], [cache rows][kd] x2
    int64_t units;              // m * U
    int64_t items;              // m * groups: work items of the vector path (G consecutive heads of one token)
    uint32_t groups;            // work items per token
    FastDiv gdiv;               // division by groups
    int64_t stride, qd, kd;
    uint32_t U, heads, kv_heads;  // U = heads + 2 kv_heads
    uint32_t hd, pos0;
    uint32_t ring;              // 0: cache row pos0 + i
    FastDiv udiv, rdiv;         // division by U and by ring
    float eps;
};

// Destination and head-norm weight of unit u (row, head h of U) of the general path: q heads, then k heads, then
// v heads.
struct Unit {
    uint32_t row;
    int kind;  // 0 q, 1 k, 2 v
    float *dst;
    const float *nw;
};

__device__ __forceinline__ Unit unit_of(const QkvRopeArgs &a, uint32_t u) {
    Unit t;
    t.row = a.udiv.div(u);
    const uint32_t h = u - t.row * a.U;
    const uint32_t pos = a.pos0 + t.row;
    const int64_t slot = a.ring ? int64_t(a.rdiv.mod(pos)) : int64_t(pos);
    if (h < a.heads) {
        t.kind = 0;
        t.dst = a.q + int64_t(t.row) * a.qd + int64_t(h) * a.hd;
        t.nw = a.qn;
    } else if (h < a.heads + a.kv_heads) {
        t.kind = 1;
        t.dst = a.kc + slot * a.kd + int64_t(h - a.heads) * a.hd;
        t.nw = a.kn;
    } else {
        t.kind = 2;
        t.dst = a.vc + slot * a.kd + int64_t(h - a.heads - a.kv_heads) * a.hd;
        t.nw = nullptr;
    }
    return t;
}

// Unit u's source: head h of row `row` in the fused projection, which lies at offset h * hd of the row for every
// kind (q heads, then k heads, then v heads, as qkvsplit.comp:16-18).
__device__ __forceinline__ const float *unit_src(const QkvRopeArgs &a, uint32_t u) {
    const uint32_t row = a.udiv.div(u);
    return a.qkv + int64_t(row) * a.stride + int64_t(u - row * a.U) * a.hd;
}

template <int E>
__device__ __forceinline__ void load_lane(const float *p, float (&v)[E]) {
    if constexpr (E == 2) {
        const float2 t = __ldcs(reinterpret_cast<const float2 *>(p));
        v[0] = t.x;
        v[1] = t.y;
    } else {
#pragma unroll
        for (int k = 0; k < E / 4; ++k) {
            const float4 t = __ldcs(reinterpret_cast<const float4 *>(p) + k);
            v[4 * k] = t.x, v[4 * k + 1] = t.y, v[4 * k + 2] = t.z, v[4 * k + 3] = t.w;
        }
    }
}
template <int E>
__device__ __forceinline__ void load_param(const float *p, float (&v)[E]) {
    if constexpr (E == 2) {
        const float2 t = __ldg(reinterpret_cast<const float2 *>(p));
        v[0] = t.x;
        v[1] = t.y;
    } else {
#pragma unroll
        for (int k = 0; k < E / 4; ++k) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(p) + k);
            v[4 * k] = t.x, v[4 * k + 1] = t.y, v[4 * k + 2] = t.z, v[4 * k + 3] = t.w;
        }
    }
}
template <int E>
__device__ __forceinline__ void store_lane(float *p, const float (&v)[E]) {
    if constexpr (E == 2) {
        *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int k = 0; k < E / 4; ++k) reinterpret_cast<float4 *>(p)[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    }
}

// Vector path (hd = 32 E): one work item = G consecutive heads (4 KB of the projection) of one token, all G loads in
// flight before the first head is finished. Lane l holds elements E l .. E l + E - 1 of a head; the rotation partners
// of its elements sit in lane l ^ 16 at the same register index, and its cos/sin pairs (indices p = E (l & 15) + j)
// are the same for every head of the token, so they are loaded once per item; the head-norm weights once per warp.
template <int E>
__global__ void __launch_bounds__(kThreads) qkv_rope_kernel(QkvRopeArgs a) {
    constexpr int HD = 32 * E, G = 32 / E;
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const bool second = lane >= 16;  // this lane holds b = x[p + hd/2]; its partner holds a = x[p]
    float qw[E], kw[E];
    if (a.qn) load_param<E>(a.qn + lane * E, qw);
    if (a.kn) load_param<E>(a.kn + lane * E, kw);
    const int64_t gw = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t nw = int64_t(gridDim.x) * kWarps;
    for (int64_t it = gw; it < a.items; it += nw) {
        const uint32_t row = a.gdiv.div(uint32_t(it));
        const uint32_t h0 = (uint32_t(it) - row * a.groups) * G;
        const uint32_t nu = a.U - h0 < uint32_t(G) ? a.U - h0 : uint32_t(G);
        const float *src = a.qkv + int64_t(row) * a.stride + int64_t(h0) * HD + lane * E;
        float x[G][E];
#pragma unroll
        for (int j = 0; j < G; ++j)
            if (uint32_t(j) < nu) load_lane<E>(src + j * HD, x[j]);
        float cs[2 * E];
        const float *csr = a.cs + (int64_t(row) * (16 * E) + (lane & 15) * E) * 2;
#pragma unroll
        for (int k = 0; k < E / 2; ++k) {
            const float4 c4 = __ldg(reinterpret_cast<const float4 *>(csr) + k);
            cs[4 * k] = c4.x, cs[4 * k + 1] = c4.y, cs[4 * k + 2] = c4.z, cs[4 * k + 3] = c4.w;
        }
        const uint32_t pos = a.pos0 + row;
        const int64_t slot = a.ring ? int64_t(a.rdiv.mod(pos)) : int64_t(pos);
        float *qrow = a.q + int64_t(row) * a.qd + lane * E;
        float *krow = a.kc + slot * a.kd + lane * E;
        float *vrow = a.vc + slot * a.kd + lane * E;
#pragma unroll
        for (int j = 0; j < G; ++j) {
            if (uint32_t(j) >= nu) break;
            const uint32_t h = h0 + j;
            if (h >= a.heads + a.kv_heads) {  // v head: copied to the V cache row
                store_lane<E>(vrow + int64_t(h - a.heads - a.kv_heads) * HD, x[j]);
                continue;
            }
            const bool is_q = h < a.heads;
            float *dst = is_q ? qrow + int64_t(h) * HD : krow + int64_t(h - a.heads) * HD;
            if (is_q ? a.qn != nullptr : a.kn != nullptr) {
                // vox::rmsnorm over the head (kernels.cpp:707-712); hd is a power of two here, so ss * (1/hd) is ss / hd
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < E; ++e) ss = fmaf(x[j][e], x[j][e], ss);
                const float inv = rsqrtf(fmaf(warp_sum(ss), 1.0f / float(HD), a.eps));
#pragma unroll
                for (int e = 0; e < E; ++e) x[j][e] = __fmul_rn(is_q ? qw[e] : kw[e], __fmul_rn(x[j][e], inv));
            }
            float o[E];
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const float other = __shfl_xor_sync(0xffffffffu, x[j][e], 16);
                const float c = cs[2 * e], sn = cs[2 * e + 1];
                // kernels.cpp:753-754: p[i] = a*c - b*s; p[i+half] = b*c + a*s
                o[e] = second ? __fadd_rn(__fmul_rn(x[j][e], c), __fmul_rn(other, sn))
                              : __fsub_rn(__fmul_rn(x[j][e], c), __fmul_rn(other, sn));
            }
            store_lane<E>(dst, o);
        }
    }
}

// General path (any even hd, any 4-byte alignment): one warp per unit through a per-warp shared buffer of hd floats.
__global__ void __launch_bounds__(kThreads) qkv_rope_general(QkvRopeArgs a) {
    pdl_enter();
    extern __shared__ float wbuf[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *v = wbuf + int64_t(warp) * a.hd;
    const int64_t gw = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t nw = int64_t(gridDim.x) * kWarps;
    const uint32_t hd = a.hd, half = hd / 2;
    for (int64_t u = gw; u < a.units; u += nw) {
        const Unit t = unit_of(a, uint32_t(u));
        const float *src = unit_src(a, uint32_t(u));
        if (t.kind == 2) {
            for (uint32_t e = lane; e < hd; e += 32) t.dst[e] = src[e];
            continue;
        }
        float ss = 0.f;
        for (uint32_t e = lane; e < hd; e += 32) {
            const float x = src[e];
            v[e] = x;
            ss = fmaf(x, x, ss);
        }
        __syncwarp();
        if (t.nw) {
            ss = warp_sum(ss);
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(hd)), a.eps)));
            for (uint32_t e = lane; e < hd; e += 32) v[e] = __fmul_rn(t.nw[e], __fmul_rn(v[e], inv));
            __syncwarp();
        }
        const float *csr = a.cs + int64_t(t.row) * half * 2;
        for (uint32_t p = lane; p < half; p += 32) {
            const float c = csr[2 * p], s = csr[2 * p + 1], x0 = v[p], x1 = v[p + half];
            t.dst[p] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            t.dst[p + half] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
        }
        __syncwarp();  // the buffer is reused by the warp's next unit
    }
}

// cs[(i * half + p) * 2] = cos(f), + 1 = sin(f), f = inv_freq[p] * float(pos0 + i) (gpu_vulkan.cpp:855-860).
__global__ void __launch_bounds__(kThreads) rope_table_kernel(const float *inv_freq, int64_t half, int64_t pos0, int64_t m,
                                                              float2 *cs) {
    pdl_enter();
    const int64_t n = m * half;
    for (int64_t k = int64_t(blockIdx.x) * kThreads + threadIdx.x; k < n; k += int64_t(gridDim.x) * kThreads) {
        const int64_t i = k / half, p = k - i * half;
        const float f = __fmul_rn(__ldg(inv_freq + p), float(pos0 + i));
        float s, c;
        sincosf(f, &s, &c);
        cs[k] = make_float2(c, s);
    }
}

bool aligned_to(const void *p, uintptr_t b) { return (reinterpret_cast<uintptr_t>(p) & (b - 1)) == 0; }

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_rope_table(const float *inv_freq, int64_t half, int64_t pos0, int64_t m, float *cs, void *stream) {
    VOX_REQUIRE(half > 0 && m >= 0 && pos0 >= 0, "vox_cuda_rope_table: bad shape");
    if (m == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(inv_freq && cs, "vox_cuda_rope_table: NULL pointer");
    VOX_REQUIRE(aligned_to(cs, 8), "vox_cuda_rope_table: cs must be 8-byte aligned");
    const int g = grid_for(m * half, kThreads, 8);
    launch_k(rope_table_kernel, g, kThreads, 0, reinterpret_cast<cudaStream_t>(stream), inv_freq, half, pos0, m,
             reinterpret_cast<float2 *>(cs));
    return check_launch("vox_cuda_rope_table");
}

int vox_cuda_qkv_rope(const float *qkv, const float *q_norm_w, const float *k_norm_w, const float *cs, float *q, float *k_cache,
                      float *v_cache, int64_t m, int64_t heads, int64_t kv_heads, int64_t hd, int64_t pos0, int64_t ring, float eps,
                      void *stream) {
    VOX_REQUIRE(m >= 0 && heads > 0 && kv_heads > 0 && hd > 0 && hd % 2 == 0 && pos0 >= 0 && ring >= 0,
                "vox_cuda_qkv_rope: bad shape (head_dim must be even)");
    if (m == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(qkv && cs && q && k_cache && v_cache, "vox_cuda_qkv_rope: NULL pointer");
    VOX_REQUIRE(ring == 0 || m <= ring, "vox_cuda_qkv_rope: more tokens than ring slots in one call (a slot would be written twice)");
    const int64_t U = heads + 2 * kv_heads;
    VOX_REQUIRE(m * U < (int64_t(1) << 32) && pos0 + m < (int64_t(1) << 32) && ring < (int64_t(1) << 32) && hd <= 4096,
                "vox_cuda_qkv_rope: sizes out of range");
    QkvRopeArgs a;
    a.qkv = qkv, a.qn = q_norm_w, a.kn = k_norm_w, a.cs = cs, a.q = q, a.kc = k_cache, a.vc = v_cache;
    a.units = m * U;
    a.qd = heads * hd, a.kd = kv_heads * hd, a.stride = a.qd + 2 * a.kd;
    a.U = uint32_t(U), a.heads = uint32_t(heads), a.kv_heads = uint32_t(kv_heads), a.hd = uint32_t(hd), a.pos0 = uint32_t(pos0);
    a.ring = uint32_t(ring);
    a.udiv = FastDiv(uint32_t(U));
    a.rdiv = FastDiv(uint32_t(ring > 0 ? ring : 1));
    a.eps = eps;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int E = int(hd / 32);
    const bool al16 = aligned16(qkv) && aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(cs) &&
                      (!q_norm_w || aligned16(q_norm_w)) && (!k_norm_w || aligned16(k_norm_w));
    const bool vec = hd % 32 == 0 && (E == 2 || E == 4 || E == 8) && al16;
    if (vec) {
        const uint32_t G = uint32_t(32 / E);
        a.groups = uint32_t((U + G - 1) / G);
        a.items = m * int64_t(a.groups);
        a.gdiv = FastDiv(a.groups);
        auto kern = E == 2 ? qkv_rope_kernel<2> : E == 4 ? qkv_rope_kernel<4> : qkv_rope_kernel<8>;
        launch_k(kern, balanced_grid(a.items, kWarps, resident_blocks((const void *)kern, kThreads, 0)), kThreads, 0, st, a);
    } else {
        const int64_t want = (a.units + kWarps - 1) / kWarps;
        const size_t smem = size_t(kWarps) * size_t(hd) * sizeof(float);
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(qkv_rope_general, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
            return check_launch("vox_cuda_qkv_rope");
        const int cap = resident_blocks((const void *)qkv_rope_general, kThreads, smem);
        launch_k(qkv_rope_general, int(want < cap ? want : cap), kThreads, smem, st, a);
    }
    return check_launch("vox_cuda_qkv_rope");
}

}  // extern "C"
