// F5-TTS DiT step on the device, captured as one CUDA graph (vox_cuda_f5_*).
//
// The step is Vox's gpu_f5_step (gpu_f5.cpp:273-332; CPU F5Model::dit_forward, f5.cpp:563-724): the input embedding
// (in_proj, then two grouped position convolutions with Mish, as im2col + batched GEMMs), then for each block an ada GEMV, the modulated LayerNorm, the q/k/v projections, RoPE, unmasked attention per sequence and
// head, the output projection and gated residual, then the MLP (ff1, GELU-tanh, ff2) and its gated residual; at the
// end the final modulation and the output projection. The elementwise and normalisation steps are this library's
// kernels (vox_cuda_adaln with no gate, vox_cuda_gated_add, vox_cuda_gelu, vox_cuda_softmax_rows) plus the RoPE kernel
// below; the projections and the two attention products are cuBLAS GEMMs (f32, or on the tensor cores with TF32 or
// bf16 inputs and f32 accumulation). In the f32 and TF32 modes attention materialises the score matrix of one
// sequence at a time ([heads][frames][frames] f32) and normalises it in place with the row softmax; in the bf16 mode
// (dim_head 64) one fused kernel computes it from the bf16 q|k|v projection without writing the scores (tcgen05
// bf16 products accumulated in tensor memory, online softmax).
//
// The plan records the whole step once eagerly (kernel selection, first-use attributes), then again under stream
// capture; a run is one cudaGraphLaunch. All buffers are the plan's, so the graph's pointers never change.
#include <cublas_v2.h>

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <string>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "sfu.cuh"
#include "gemm.cuh"
#include "tc.cuh"
#include "rows.cuh"

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

// ------------------------------------------------------------------ input embedding (grouped position convolutions)

// Conv weights from PyTorch's [cout][cig][K] into [cout][K][cig] (the order of the im2col columns), f32 or bf16 (RN),
// once at create.
template <typename TO>
__global__ void __launch_bounds__(256) f5_conv_reorder_kernel(const float *w, TO *wr, uint32_t n, uint32_t cig, uint32_t K) {
    pdl_enter();
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
        const uint32_t i = e % cig, t = e / cig, k = t % K, o = t / K;  // e = (o K + k) cig + i
        wr[e] = TO(w[(size_t(o) * cig + i) * K + k]);
    }
}

// im2col of x [B][T][cin] (f32) for a grouped convolution with zero padding K/2: col [B][groups][T][K cig] with column
// k cig + i = x[t + k - K/2][g cig + i] (zero outside the sequence), in f32 or rounded to bf16 (RN); VW channels per
// thread (4 when cig % 4 == 0, else 1).
template <int VW, bool BF16>
__global__ void __launch_bounds__(256) f5_im2col_kernel(const float *x, void *col, uint32_t items, uint32_t T, uint32_t cin,
                                                        uint32_t groups, uint32_t K) {
    pdl_enter();
    using V = typename std::conditional<VW == 4, float4, float>::type;
    const uint32_t cq = cin / groups / VW;  // items per tap of one group
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < items; e += gridDim.x * blockDim.x) {
        const uint32_t iq = e % cq, r1 = e / cq, k = r1 % K, r2 = r1 / K;  // e = ((sg T + t) K + k) cq + iq
        const uint32_t t = r2 % T, sg = r2 / T, g = sg % groups, sq = sg / groups;
        const int tt = int(t) + int(k) - int(K / 2);
        V v{};
        if (tt >= 0 && tt < int(T)) v = reinterpret_cast<const V *>(x)[(size_t(sq) * T + uint32_t(tt)) * (cin / VW) + g * cq + iq];
        if constexpr (!BF16) {
            reinterpret_cast<V *>(col)[e] = v;
        } else if constexpr (VW == 4) {
            reinterpret_cast<uint2 *>(col)[e] = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
        } else {
            reinterpret_cast<__nv_bfloat16 *>(col)[e] = __float2bfloat16_rn(v);
        }
    }
}

// The bf16 im2col with 8 columns (16 bytes) an item: item e of row r = (sq groups + g) T + t is tap k = j / (cig / 8),
// column block q = j % (cig / 8) (j = e % (K cig / 8)), read as two float4 of x[sq][t + k - K/2][g cig + 8 q ..] (zero
// past the sequence) and written as one uint4. The divisions by the launch's invariants use FastDiv; kIm2colUnroll
// items a thread and pass are loaded before any is stored.
constexpr int kIm2colUnroll = 4;
__global__ void __launch_bounds__(256) f5_im2col8_kernel(const float *x, uint4 *col, uint32_t items, uint32_t T, uint32_t cin,
                                                         uint32_t cig, uint32_t K, FastDiv per_row, FastDiv per_tap, FastDiv tdiv,
                                                         FastDiv gdiv) {
    pdl_enter();
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t e0 = blockIdx.x * blockDim.x + threadIdx.x; e0 < items; e0 += kIm2colUnroll * stride) {
        float4 a[kIm2colUnroll], b[kIm2colUnroll];
#pragma unroll
        for (int u = 0; u < kIm2colUnroll; ++u) {
            const uint32_t e = e0 + u * stride;
            a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e < items) {
                const uint32_t row = per_row.div(e), j = e - row * per_row.d;
                const uint32_t k = per_tap.div(j), q = j - k * per_tap.d;
                const uint32_t sg = tdiv.div(row), t = row - sg * T;
                const uint32_t sq = gdiv.div(sg), g = sg - sq * gdiv.d;
                const int tt = int(t) + int(k) - int(K / 2);
                if (tt >= 0 && tt < int(T)) {
                    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t(sq) * T + uint32_t(tt)) * cin + g * cig + 8 * q);
                    a[u] = src[0];
                    b[u] = src[1];
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kIm2colUnroll; ++u) {
            const uint32_t e = e0 + u * stride;
            if (e < items)
                col[e] = make_uint4(pack_bf16(a[u].x, a[u].y), pack_bf16(a[u].z, a[u].w), pack_bf16(b[u].x, b[u].y), pack_bf16(b[u].z, b[u].w));
        }
    }
}

// mish(x) = x tanh(softplus(x)), softplus = x past 20 (f5.cpp:97-100), with the accurate CUDA functions.
__device__ __forceinline__ float mish_f(float x) {
    const float sp = x > 20.f ? x : log1pf(expf(x));
    return x * tanhf(sp);
}
// v = mish(y + bias[col]); y = v (res NULL) or res += v (rounded add); n elements of rows of D.
__global__ void __launch_bounds__(256) f5_bias_mish_kernel(float *y, const float *bias, float *res, uint32_t n, uint32_t D) {
    pdl_enter();
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
        const float v = mish_f(__fadd_rn(y[e], bias ? bias[e % D] : 0.f));
        if (res) res[e] = __fadd_rn(res[e], v);
        else y[e] = v;
    }
}

// ------------------------------------------------------------------ fused attention (bf16 math mode, dim_head 64)

// The bf16 q|k|v projection qkv [rows][3 inner] in place: + bias (f32 [3 inner]), then RoPE on the q and k of heads
// < rope_heads (each pair widened to f32 and rotated with the rounding of the CPU loop, f5.cpp:696-701), rounded back
// to bf16 (RN); the bias comes first, as matmul adds it (kernels.hpp:83). Eight columns (16 bytes) per thread, hd % 8 == 0.
__global__ void __launch_bounds__(256) f5_qkv_bias_rope_kernel(uint4 *qkv, const float *bias, const float2 *cs, uint32_t octs,
                                                               uint32_t frames, uint32_t half, uint32_t rope_heads, uint32_t hd,
                                                               uint32_t inner) {
    pdl_enter();
    const uint32_t stride = gridDim.x * blockDim.x, row_octs = 3 * inner / 8;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < octs; i += stride) {
        const uint32_t r = i / row_octs, c = 8 * (i % row_octs);
        const uint32_t part = c / inner, ci = c % inner, head = ci / hd;
        uint4 w = qkv[i];
        uint32_t *wp = &w.x;
        const float4 b0 = *reinterpret_cast<const float4 *>(bias + c), b1 = *reinterpret_cast<const float4 *>(bias + c + 4);
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float x[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            x[2 * k] = __fadd_rn(__uint_as_float(wp[k] << 16), bb[2 * k]);
            x[2 * k + 1] = __fadd_rn(__uint_as_float(wp[k] & 0xFFFF0000u), bb[2 * k + 1]);
        }
        if (part < 2 && head < rope_heads) {
            const float4 *c4 = reinterpret_cast<const float4 *>(cs + size_t(r % frames) * half + (ci % hd) / 2);
            const float4 ca = c4[0], cb = c4[1];
            const float cc[4] = {ca.x, ca.z, cb.x, cb.z}, ss[4] = {ca.y, ca.w, cb.y, cb.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float x0 = x[2 * k], x1 = x[2 * k + 1];
                x[2 * k] = __fsub_rn(__fmul_rn(x0, cc[k]), __fmul_rn(x1, ss[k]));
                x[2 * k + 1] = __fadd_rn(__fmul_rn(x1, cc[k]), __fmul_rn(x0, ss[k]));
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) wp[k] = pack_bf16(x[2 * k], x[2 * k + 1]);
        qkv[i] = w;
    }
}

// ff [rows][F] bf16 in place: gelu_tanh(x + bias) (bias f32 [F]); eight columns per thread, F % 8 == 0.
__global__ void __launch_bounds__(256) f5_bias_gelu_kernel(uint4 *ff, const float *bias, uint32_t octs, uint32_t F) {
    pdl_enter();
    const uint32_t stride = gridDim.x * blockDim.x, row_octs = F / 8;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < octs; i += stride) {
        const uint32_t c = 8 * (i % row_octs);
        uint4 w = ff[i];
        uint32_t *wp = &w.x;
        const float4 b0 = *reinterpret_cast<const float4 *>(bias + c), b1 = *reinterpret_cast<const float4 *>(bias + c + 4);
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 v = gelu_tanh_f2(make_float2(__fadd_rn(__uint_as_float(wp[k] << 16), bb[2 * k]),
                                                      __fadd_rn(__uint_as_float(wp[k] & 0xFFFF0000u), bb[2 * k + 1])));
            wp[k] = pack_bf16(v.x, v.y);
        }
        ff[i] = w;
    }
}

constexpr int kFaHd = 64;     // head dimension of the fused kernel

// A tile of rows of 64 bf16 (128-byte rows) in shared memory: the 16-byte chunk c of row r sits at chunk c ^ (r % 8)
// (the 128-byte swizzle of the tensor cores' shared-memory operands; 8 consecutive rows' chunk c in 8 bank groups).
__device__ __forceinline__ uint32_t fa_off(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

// cp.async of one 16-byte chunk; src_bytes 0 fills the chunk with zeros (rows past the sequence end).
__device__ __forceinline__ void cp16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// ------------------------------------------------------------------ fused attention on the 5th-generation tensor cores

// softmax(q k^T * scale) v for one sequence and head, 128 query rows per CTA, on tcgen05: S = Q K^T (M 128, N 64 keys, K 64) and each tile's
// P V (M 128, N 64, K 64 keys) are accumulated in tensor memory (TMEM lane = query row, f32), their operands read
// from shared memory through matrix descriptors. Q [128 rows][64 bf16], K and V tiles [64 keys][64 bf16] and P
// [128 rows][64 keys] sit in the 128-byte swizzle (fa_off: 16-byte chunk c of row r at chunk c ^ (r % 8)), which is
// the canonical K-major SW128 layout for Q, K, P and the MN-major SW128 layout for V (the head dimension is V's N).
// Thread t of the 4 warps owns query row t: it reads its S row from TMEM (two passes of 32 columns: the maximum, then
// 2^(s scale log2e - max), rounded to bf16 into P), and after each tile's P V adds that tile's O row to its f32
// accumulator rescaled by the online-softmax factor. One thread issues the MMAs; their completion arrives on
// mbarriers (tcgen05.commit); every wait is bounded. K and V of the next tile load by cp.async during this tile.
// 65 KB of shared memory and 128 TMEM columns a CTA: three CTAs share an SM, so one's softmax overlaps another's MMAs.
constexpr int kTcRows = 128;
constexpr int kTcKeys = 64;
constexpr int kTcThreads = 128;
constexpr uint32_t kTcQ = 128 * 128;     // Q and P tiles, [128][64] bf16, bytes
constexpr uint32_t kTcKV = 64 * 128;     // K and V tiles, [64][64] bf16
constexpr uint32_t kTcCols = 128;        // TMEM columns: S 0..63, P V 64..127
constexpr size_t kTcSmem = 2 * size_t(kTcQ) + 4 * size_t(kTcKV) + 1024 + 128;  // Q, P, K[2], V[2]; alignment; barriers

// Instruction descriptors of the two products (M 128, N 64): S = Q K^T with both operands K-major, and P V with V
// MN-major.
constexpr uint32_t kIdescS = umma_idesc_bf16(128, 64);
constexpr uint32_t kIdescO = umma_idesc_bf16(128, 64, true);

// Stages rows [row0, row0 + ROWS) of a head's 64 columns (global row stride ld bf16) into a swizzled tile; rows at
// or past n are zero-filled. 8 chunks a row, ROWS / 16 per thread.
template <int ROWS, int THREADS = kTcThreads>
__device__ __forceinline__ void tc_stage(uint32_t tile, const __nv_bfloat16 *g, int row0, int n, int ld) {
#pragma unroll
    for (int u = 0; u < ROWS * 8 / THREADS; ++u) {
        const int idx = threadIdx.x + u * THREADS, r = idx >> 3, c = idx & 7;
        const int gr = row0 + r;
        cp16(tile + fa_off(r, c), g + size_t(gr < n ? gr : n - 1) * ld + c * 8, gr < n ? 16u : 0u);
    }
}

__global__ void __launch_bounds__(kTcThreads, 3) f5_flash_tc_kernel(const __nv_bfloat16 *qb, const __nv_bfloat16 *kb,
                                                                    const __nv_bfloat16 *vb, __nv_bfloat16 *at, int n, int ld_in,
                                                                    int inner, float scale_log2) {
    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sQ = smem_addr(smem), sP = sQ + kTcQ, sK = sQ + 2 * kTcQ, sV = sK + 2 * kTcKV;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + 2 * kTcQ + 4 * kTcKV);  // [0] S done, [1] P V done
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + 2 * kTcQ + 4 * kTcKV + 16);
    const int warp = threadIdx.x >> 5, row = threadIdx.x;
    const int q0 = blockIdx.x * kTcRows, head = blockIdx.y;
    const size_t seq = size_t(blockIdx.z) * size_t(n) * size_t(ld_in) + size_t(head) * kFaHd;
    const __nv_bfloat16 *Q = qb + seq, *K = kb + seq, *V = vb + seq;
    const int ntiles = (n + kTcKeys - 1) / kTcKeys;
    pdl_enter();  // the previous grid (and the tensor memory it held) is complete
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init_fence();
    }
    if (warp == 0) {
        tmem_alloc(tslot, kTcCols);
    }
    tc_stage<kTcRows>(sQ, Q, q0, n, ld_in);
    tc_stage<kTcKeys>(sK, K, 0, n, ld_in);
    tc_stage<kTcKeys>(sV, V, 0, n, ld_in);
    asm volatile("cp.async.commit_group;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);  // this warp's 32 lanes
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    float mrow = -INFINITY, lrow = 0.f;
    bool ok = true;
    // tile 0's K and V, then its S product; each iteration below issues tile kt's P V together with tile kt + 1's S
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // this thread's tile writes, visible to the MMA
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 16 of the 64 head dimensions a step: 32 bytes along the swizzled rows
            umma_bf16(tmem, umma_desc(sQ + 32 * k, 16, 1024), umma_desc(sK + 32 * k, 16, 1024), kIdescS, k > 0);
        umma_commit(&bar[0]);
    }
    for (int kt = 0; kt < ntiles; ++kt) {  // every thread runs every iteration's barrier, ok or not
        const int buf = kt & 1;
        if (kt + 1 < ntiles) {  // the other buffers' last readers (tile kt - 1's products) have completed
            tc_stage<kTcKeys>(sK + (buf ^ 1) * kTcKV, K, (kt + 1) * kTcKeys, n, ld_in);
            tc_stage<kTcKeys>(sV + (buf ^ 1) * kTcKV, V, (kt + 1) * kTcKeys, n, ld_in);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        ok = ok && mbar_wait_warp(&bar[0], uint32_t(kt & 1));  // a wait that gives up sets the device error flag
        tc_fence_after();
        float alpha = 1.f;
        if (ok) {
            const int key0 = kt * kTcKeys;
            const bool full = key0 + kTcKeys <= n;  // else keys past the sequence end take no weight
            // the tile's S row: both 32-column loads in flight, one wait
            uint32_t r[kTcKeys];
            tmem_ld32(trow, *reinterpret_cast<uint32_t(*)[32]>(r));
            tmem_ld32(trow + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
            tmem_wait_ld();
            if (!full) {  // keys past the sequence end: -inf scores, so their weights are 2^-inf = 0
#pragma unroll
                for (int i = 0; i < kTcKeys; ++i)
                    if (key0 + i >= n) r[i] = __float_as_uint(-INFINITY);
            }
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < kTcKeys; i += 2) mx = fmaxf(mx, fmaxf(__uint_as_float(r[i]), __uint_as_float(r[i + 1])));
            const float mnew = fmaxf(mrow, mx * scale_log2);
            alpha = ex2_approx(mrow - mnew);
            // P = 2^(s scale log2e - max) in bf16 into P (tile kt - 1's P V has read it), and the row sum of the
            // unrounded values
            float sum = 0.f;
            const float2 sl2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-mnew, -mnew);
#pragma unroll
            for (int ch = 0; ch < kTcKeys / 8; ++ch) {  // 8 keys (one 16-byte chunk) a step
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = 8 * ch + 2 * e;
                    const float2 a = fma2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), sl2, nm2);
                    const float p0 = ex2_approx(a.x), p1 = ex2_approx(a.y);
                    sum += p0 + p1;
                    w[e] = pack_bf16(p0, p1);
                }
                const uint32_t dst = sP + fa_off(row, ch);  // key chunk 0..7 of the row
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]) : "memory");
            }
            lrow = lrow * alpha + sum;
            mrow = mnew;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");          // tile kt + 1's K and V
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P and the tile, visible to the MMA
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x == 0 && ok) {
            tc_fence_after();
            const uint32_t tV = sV + buf * kTcKV, tK1 = sK + (buf ^ 1) * kTcKV;
#pragma unroll
            for (int k = 0; k < 4; ++k)  // 16 keys a step: P along its swizzled rows, V by 16 rows (2048 bytes)
                umma_bf16(tmem + 64, umma_desc(sP + 32 * k, 16, 1024), umma_desc(tV + 2048 * k, 16384, 1024), kIdescO, k > 0);
            umma_commit(&bar[1]);
            if (kt + 1 < ntiles) {  // the next tile's S: every thread has read this tile's S before the barrier
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    umma_bf16(tmem, umma_desc(sQ + 32 * k, 16, 1024), umma_desc(tK1 + 32 * k, 16, 1024), kIdescS, k > 0);
                umma_commit(&bar[0]);
            }
        }
        ok = ok && mbar_wait_warp(&bar[1], uint32_t(kt & 1));
        tc_fence_after();
        if (ok) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t r[32];
                tmem_ld32(trow + 64 + 32 * c, r);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float2 v = fma2(make_float2(o[32 * c + i], o[32 * c + i + 1]), make_float2(alpha, alpha),
                                          make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])));
                    o[32 * c + i] = v.x;
                    o[32 * c + i + 1] = v.y;
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (ok && q0 + row < n) {
        const float inv = 1.0f / lrow;
        uint4 *dst = reinterpret_cast<uint4 *>(at + (size_t(blockIdx.z) * size_t(n) + size_t(q0 + row)) * inner + size_t(head) * kFaHd);
#pragma unroll
        for (int c = 0; c < 8; ++c)
            dst[c] = make_uint4(pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv), pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                                pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv), pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
    }
}

// ------------------------------------------------------------------ bf16 pipeline helpers

// The same attention with two threads a query row: 8 warps, warp w reads TMEM lanes 32 (w % 4) .. (its 32 query rows)
// and takes keys 32 h .. 32 h + 31 of each S tile and head dimensions 32 h .. 32 h + 31 of each P V tile, h = w / 4.
// The two halves of a row exchange their partial maxima through shared memory (a named barrier per pair of warps)
// and add their partial row sums once at the end; both halves apply the same running maximum, so their sums and
// output columns share one scale. Each thread's serial softmax chain is half as long (and split into four independent
// max and sum chains) and twice as many warps share an SM as with one thread a row. Warp 0 issues the MMAs through an
// elected lane (operands warp-uniform). Measured against the alternatives on B200 (F5 base, 2 x 1024 frames, 16
// heads): 28.9 us a launch against 31.2 us for one thread a row; keeping two S and two P V buffers in tensor memory
// so that P V of a tile is waited for one tile later measured 33.5 us, and the same with a ninth warp issuing the
// MMAs (no CTA-wide barrier in the loop) 37.0 us. In the step (same box, 22 launches): the next tile's S issued before
// this tile's P V, P V folded into the output after the next tile's exponentials and K / V in three buffers took the
// step from 2.200 to 2.272 ms; a quarter of the exponentials from a cubic on the FMA pipe (beside the MUFU ex2), from
// 2.203 to 2.215 ms.
constexpr int kTc2Threads = 256;
constexpr size_t kTc2Smem = kTcSmem + 2 * 128 * sizeof(float);  // + the partial maxima / sums of the two halves

__global__ void __launch_bounds__(kTc2Threads, 2) f5_flash_tc2_kernel(const __nv_bfloat16 *qb, const __nv_bfloat16 *kb,
                                                                      const __nv_bfloat16 *vb, __nv_bfloat16 *at, int n, int ld_in,
                                                                      int inner, float scale_log2) {
    extern __shared__ uint8_t tc2_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc2_smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sQ = smem_addr(smem), sP = sQ + kTcQ, sK = sQ + 2 * kTcQ, sV = sK + 2 * kTcKV;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + 2 * kTcQ + 4 * kTcKV);  // [0] S done, [1] P V done, [2] drain
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + 2 * kTcQ + 4 * kTcKV + 32);
    float *red = reinterpret_cast<float *>(smem + 2 * kTcQ + 4 * kTcKV + 128);  // [2][128]: half h's value for row r
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, quad = warp & 3, half = warp >> 2;
    const int row = 32 * quad + lane;  // query row within the tile
    const int q0 = blockIdx.x * kTcRows, head = blockIdx.y;
    const size_t seq = size_t(blockIdx.z) * size_t(n) * size_t(ld_in) + size_t(head) * kFaHd;
    const __nv_bfloat16 *Q = qb + seq, *K = kb + seq, *V = vb + seq;
    const int ntiles = (n + kTcKeys - 1) / kTcKeys;
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory"); };  // the row's two warps
    pdl_enter();  // the previous grid (and the tensor memory it held) is complete
    if (threadIdx.x == 0) {
        for (int i = 0; i < 3; ++i) mbar_init(&bar[i], 1);
        mbar_init_fence();
    }
    if (warp == 0) tmem_alloc(tslot, kTcCols);
    tc_stage<kTcRows, kTc2Threads>(sQ, Q, q0, n, ld_in);
    tc_stage<kTcKeys, kTc2Threads>(sK, K, 0, n, ld_in);
    tc_stage<kTcKeys, kTc2Threads>(sV, V, 0, n, ld_in);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16);  // this warp's 32 lanes
    float o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = 0.f;
    float mrow = -INFINITY, lrow = 0.f;
    bool ok = true;
    if (warp == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
            umma_bf16_warp(tmem, umma_desc(sQ + 32 * k, 16, 1024), umma_desc(sK + 32 * k, 16, 1024), kIdescS, k > 0);
        umma_commit_warp(&bar[0]);
    }
    for (int kt = 0; kt < ntiles; ++kt) {  // every thread runs every iteration's barriers, ok or not
        const int buf = kt & 1;
        if (kt + 1 < ntiles) {  // the other buffers' last readers (tile kt - 1's products) have completed
            tc_stage<kTcKeys, kTc2Threads>(sK + (buf ^ 1) * kTcKV, K, (kt + 1) * kTcKeys, n, ld_in);
            tc_stage<kTcKeys, kTc2Threads>(sV + (buf ^ 1) * kTcKV, V, (kt + 1) * kTcKeys, n, ld_in);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        ok = ok && mbar_wait_warp(&bar[0], uint32_t(kt & 1));
        tc_fence_after();
        float alpha = 1.f;
        uint32_t r[32];
        float mx = -INFINITY;
        if (ok) {
            const int key0 = kt * kTcKeys + 32 * half;
            tmem_ld32(trow + 32 * half, r);
            tmem_wait_ld(r);
            if (key0 + 32 > n) {  // keys past the sequence end: -inf scores, weight 2^-inf = 0
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (key0 + i >= n) r[i] = __float_as_uint(-INFINITY);
            }
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
            for (int i = 0; i < 32; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(r[i]));
            mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            red[half * 128 + row] = mx;
        }
        pair_sync();
        if (ok) {
            mx = fmaxf(mx, red[(half ^ 1) * 128 + row]);
            const float mnew = fmaxf(mrow, mx * scale_log2);
            alpha = ex2_approx(mrow - mnew);
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
            const float2 sl2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-mnew, -mnew);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {  // key chunks 4 h .. 4 h + 3 of the row (8 keys each)
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = 8 * ch + 2 * e;
                    const float2 a = fma2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), sl2, nm2);
                    const float p0 = ex2_approx(a.x), p1 = ex2_approx(a.y);
                    s4[e] += p0 + p1;
                    w[e] = pack_bf16(p0, p1);
                }
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sP + fa_off(row, 4 * half + ch)), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                             "r"(w[3])
                             : "memory");
            }
            lrow = lrow * alpha + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
            mrow = mnew;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");          // tile kt + 1's K and V
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P and the tile, visible to the MMA
        tc_fence_before();
        __syncthreads();
        if (warp == 0 && ok) {
            tc_fence_after();
            const uint32_t tV = sV + buf * kTcKV, tK1 = sK + (buf ^ 1) * kTcKV;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                umma_bf16_warp(tmem + 64, umma_desc(sP + 32 * k, 16, 1024), umma_desc(tV + 2048 * k, 16384, 1024), kIdescO, k > 0);
            umma_commit_warp(&bar[1]);
            if (kt + 1 < ntiles) {  // the next tile's S: every thread has read this tile's S before the barrier
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    umma_bf16_warp(tmem, umma_desc(sQ + 32 * k, 16, 1024), umma_desc(tK1 + 32 * k, 16, 1024), kIdescS, k > 0);
                umma_commit_warp(&bar[0]);
            }
        }
        __syncwarp();
        ok = ok && mbar_wait_warp(&bar[1], uint32_t(kt & 1));
        tc_fence_after();
        if (ok) {
            uint32_t v[32];
            tmem_ld32(trow + 64 + 32 * half, v);
            tmem_wait_ld(v);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                const float2 t = fma2(make_float2(o[i], o[i + 1]), make_float2(alpha, alpha), make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])));
                o[i] = t.x;
                o[i + 1] = t.y;
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // the row sum: this half's plus the other's (same running maximum)
    red[half * 128 + row] = lrow;
    pair_sync();
    const float ltot = lrow + red[(half ^ 1) * 128 + row];
    if (ok && q0 + row < n) {
        const float inv = 1.0f / ltot;
        uint4 *dst = reinterpret_cast<uint4 *>(at + (size_t(blockIdx.z) * size_t(n) + size_t(q0 + row)) * inner + size_t(head) * kFaHd + 32 * half);
#pragma unroll
        for (int c = 0; c < 4; ++c)
            dst[c] = make_uint4(pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv), pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                                pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv), pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {  // every MMA issued has completed (a wait above may have given up) before the memory is released
        tc_fence_after();
        umma_commit_warp(&bar[2]);
        __syncwarp();
        mbar_wait_warp(&bar[2], 0);
        tmem_dealloc(tmem, kTcCols);
    }
}

// xc [R][M + C] (bf16, RN) = [x [R][M] | cond [R][C]] (f32): the input of the in_proj GEMM; one element a thread.
__global__ void __launch_bounds__(256) f5_concat_bf16_kernel(const float *x, const float *cond, __nv_bfloat16 *xc, uint32_t n,
                                                             uint32_t M, uint32_t C) {
    pdl_enter();
    const uint32_t W = M + C;
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
        const uint32_t r = e / W, c = e - r * W;
        xc[e] = __float2bfloat16_rn(c < M ? x[size_t(r) * M + c] : cond[size_t(r) * C + (c - M)]);
    }
}

// y_l[o] = W_l[o] . x + b_l[o] for the L matrices W_l [rows][cols] (f32) of a pointer table (blockIdx.y = l): the ada
// vectors of every block from one time embedding (f5.cpp:681-682, Vox's per-block matvec). One warp per output row,
// 16-byte loads, the lanes' partial sums folded by the xor butterfly; cols % 4 == 0.
__global__ void __launch_bounds__(256) f5_gemv_f32_kernel(const float *const *W, const float *x, const float *bias, float *y,
                                                          uint32_t rows, uint32_t cols) {
    pdl_enter();
    const uint32_t l = blockIdx.y, o = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (o >= rows) return;
    const float4 *w = reinterpret_cast<const float4 *>(W[l] + size_t(o) * cols);
    const float4 *xv = reinterpret_cast<const float4 *>(x);
    float acc = 0.f;
    for (uint32_t c = lane; c < cols / 4; c += 32) {
        const float4 a = as_f4(ld_stream(w + c)), b = xv[c];
        acc = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
    }
    acc = warp_sum(acc);
    if (lane == 0) y[size_t(l) * rows + o] = acc + (bias ? bias[size_t(l) * rows + o] : 0.f);
}

// dst = bf16(src) (RN), n / 2 pairs (weights, converted once at plan creation).
__global__ void __launch_bounds__(256) f5_to_bf16_kernel(const float2 *src, uint32_t *dst, size_t pairs) {
    pdl_enter();
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < pairs; i += size_t(gridDim.x) * blockDim.x) {
        const float2 v = src[i];
        dst[i] = pack_bf16(v.x, v.y);
    }
}

// One warp per row of h [rows][D]: if delta, h += gate * (delta + dbias) (the projection's bias added first, as
// matmul does; product, then sum, each rounded: gated_add of f5.cpp:670-676); then nrm = LayerNorm(h) * (1 + scale) + shift (no affine, eps; mean and variance two-pass in f32 on
// the row in registers) rounded to bf16 for the next projection. Lane l holds columns 4 (l + 32 k), k < VPL.
// WPR warps share a row (VPL float4 a lane); their partial sums meet in shared memory across a CTA barrier.
template <int VPL, int WPR>
__global__ void __launch_bounds__(256) f5_resmod_kernel(float *h, const float *delta, const float *dbias, const float *gate,
                                                        const float *scale, const float *shift, uint2 *nrm, uint32_t rows, uint32_t D,
                                                        float eps) {
    pdl_enter();
    __shared__ float part[8][2];  // [warp][sum, squares]
    const uint32_t warp = threadIdx.x >> 5, r = (blockIdx.x * 8 + warp) / WPR, lane = (warp % WPR) * 32 + (threadIdx.x & 31);
    const bool live = r < rows;  // (no early exit: the row's warps meet at CTA barriers)
    if (WPR == 1 && !live) return;
    float4 x[VPL];
    float4 *hr = reinterpret_cast<float4 *>(h + size_t(r) * D);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const uint32_t c = lane + 32 * WPR * k;
        x[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live && 4 * c < D) {
            x[k] = hr[c];
            if (delta) {
                float4 dv = reinterpret_cast<const float4 *>(delta + size_t(r) * D)[c];
                const float4 db = reinterpret_cast<const float4 *>(dbias)[c];
                dv = make_float4(__fadd_rn(dv.x, db.x), __fadd_rn(dv.y, db.y), __fadd_rn(dv.z, db.z), __fadd_rn(dv.w, db.w));
                const float4 g = reinterpret_cast<const float4 *>(gate)[c];
                x[k] = make_float4(__fadd_rn(x[k].x, __fmul_rn(g.x, dv.x)), __fadd_rn(x[k].y, __fmul_rn(g.y, dv.y)),
                                   __fadd_rn(x[k].z, __fmul_rn(g.z, dv.z)), __fadd_rn(x[k].w, __fmul_rn(g.w, dv.w)));
                hr[c] = x[k];
            }
            sum += (x[k].x + x[k].y) + (x[k].z + x[k].w);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (WPR > 1) {
        if ((threadIdx.x & 31) == 0) part[warp][0] = sum;
        __syncthreads();
        sum = 0.f;
#pragma unroll
        for (int w = 0; w < WPR; ++w) sum += part[warp - warp % WPR + w][0];
    }
    const float mean = sum / float(D);
    float var = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
        if (live && 4 * (lane + 32 * WPR * k) < D) {
            const float a = x[k].x - mean, b = x[k].y - mean, c = x[k].z - mean, e = x[k].w - mean;
            var += (a * a + b * b) + (c * c + e * e);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    if (WPR > 1) {
        if ((threadIdx.x & 31) == 0) part[warp][1] = var;
        __syncthreads();
        var = 0.f;
#pragma unroll
        for (int w = 0; w < WPR; ++w) var += part[warp - warp % WPR + w][1];
    }
    const float inv = rsqrtf(var / float(D) + eps);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const uint32_t c = lane + 32 * WPR * k;
        if (live && 4 * c < D) {
            const float4 sc = reinterpret_cast<const float4 *>(scale)[c], sh = reinterpret_cast<const float4 *>(shift)[c];
            const float y0 = fmaf((x[k].x - mean) * inv, 1.f + sc.x, sh.x), y1 = fmaf((x[k].y - mean) * inv, 1.f + sc.y, sh.y);
            const float y2 = fmaf((x[k].z - mean) * inv, 1.f + sc.z, sh.z), y3 = fmaf((x[k].w - mean) * inv, 1.f + sc.w, sh.w);
            nrm[size_t(r) * (D / 4) + c] = make_uint2(pack_bf16(y0, y1), pack_bf16(y2, y3));
        }
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
    // f32 / TF32 path
    float *h = nullptr, *ts = nullptr, *out = nullptr, *nrm = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *at = nullptr,
          *o = nullptr, *ffb = nullptr, *s = nullptr, *ada = nullptr, *fin = nullptr;
    float2 *cs = nullptr;
    // bf16 path (bf16 math, dim_head 64, dim % 4 == 0 and <= 2048): bf16 copies of the projection weights (q|k|v fused),
    // bf16 activations into every GEMM, the fused attention, all ada vectors by one batched GEMV
    bool bf16 = false;
    float *ada_all = nullptr;
    __nv_bfloat16 *qkv_b = nullptr, *nrm_b = nullptr, *at_b = nullptr, *ff_b = nullptr;
    __nv_bfloat16 *w_qkv = nullptr, *w_o = nullptr, *w_ff1 = nullptr, *w_ff2 = nullptr, *w_proj = nullptr;
    const void **ada_ptrs = nullptr;  // device [3][depth]: W_ada[l], ts, ada_all + l 6D
    // f32 copies of every bias (zeros where the description has none), made at create: [depth][6D], [depth][3 inner],
    // [depth][D] (o), [depth][F] (ff1), [depth][D] (ff2), [2D] (norm_out), [out_dim] (proj_out)
    float *b_ada = nullptr, *b_qkv = nullptr, *b_o = nullptr, *b_ff1 = nullptr, *b_ff2 = nullptr, *b_fin = nullptr, *b_proj = nullptr;
    // tcgen05 GEMMs of the bf16 path (every K a multiple of 8): built once at create, replayed by the graph; the
    // in_proj input [x | cond] and weights in bf16
    bool tc = false;
    int tc_mask = 63;  // which GEMMs run on the tcgen05 kernel when tc (all by default)
    std::vector<GemmPlan> g_qkv, g_o, g_ff1, g_ff2;
    GemmPlan g_proj, g_in, g_conv1, g_conv2;
    __nv_bfloat16 *xc_b = nullptr, *w_in = nullptr;
    // input embedding (in_proj given): x [R][out_dim], cond [R][in_dim - out_dim], im2col scratch, reordered conv weights
    bool embed = false;
    float *xin = nullptr, *cond = nullptr, *col = nullptr, *ctmp = nullptr, *w1r = nullptr, *w2r = nullptr;
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
// The same with bf16 x and W (tensor cores, f32 accumulation) and y f32 or bf16.
int gemm_bf16(F5Plan &p, const __nv_bfloat16 *x, const __nv_bfloat16 *w, void *y, cudaDataType_t yt, int64_t R, int64_t O, int64_t I) {
    const float one = 1.0f, zero = 0.0f;
    return blas_check(cublasGemmEx(p.blas, CUBLAS_OP_T, CUBLAS_OP_N, int(O), int(R), int(I), &one, w, CUDA_R_16BF, int(I), x,
                                   CUDA_R_16BF, int(I), &zero, y, yt, int(O), CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT),
                      "gemm (bf16)");
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

constexpr int kPosGroups = 16, kPosK = 31;  // F5's position convolutions (f5.cpp:306-307)

// conv of src [R][D] (B sequences of T frames) into dst [R][D]: im2col, then per sequence one GEMM batched over the
// groups (col [T][K cig] of group g times the group's reordered weights [cog][K cig], into columns g cog of dst); in
// the bf16 mode columns and weights are bf16 (tensor cores, f32 accumulation).
int conv_pos(F5Plan &p, const float *src, const void *wr, float *dst, const GemmPlan *gp, cudaStream_t st) {
    const vox_cuda_f5_desc &d = p.d;
    const uint32_t T = uint32_t(d.frames), D = uint32_t(d.dim), cig = D / kPosGroups, J = kPosK * cig;
    const uint32_t all = uint32_t(d.batch) * kPosGroups * T * J;
    const uint32_t G = uint32_t(kPosGroups), KK = uint32_t(kPosK);
    if (p.bf16 && cig % 8 == 0) {
        const uint32_t items = all / 8;
        launch_k(f5_im2col8_kernel, grid_for((items + kIm2colUnroll - 1) / kIm2colUnroll, 256, 4), 256, 0, st, src, (uint4 *)p.col, items,
                 T, D, cig, KK, FastDiv(J / 8), FastDiv(cig / 8), FastDiv(T), FastDiv(G));
    } else if (cig % 4 == 0) {
        if (p.bf16) launch_k(f5_im2col_kernel<4, true>, grid_for(all / 4, 256, 4), 256, 0, st, src, (void *)p.col, all / 4, T, D, G, KK);
        else launch_k(f5_im2col_kernel<4, false>, grid_for(all / 4, 256, 4), 256, 0, st, src, (void *)p.col, all / 4, T, D, G, KK);
    } else {
        if (p.bf16) launch_k(f5_im2col_kernel<1, true>, grid_for(all, 256, 4), 256, 0, st, src, (void *)p.col, all, T, D, G, KK);
        else launch_k(f5_im2col_kernel<1, false>, grid_for(all, 256, 4), 256, 0, st, src, (void *)p.col, all, T, D, G, KK);
    }
    F5_TRY(check_launch("vox_cuda_f5 im2col"));
    if (gp) return gemm_run(*gp, st, "vox_cuda_f5 position convolution");  // all sequences and groups in one launch
    const float one = 1.0f, zero = 0.0f;
    const cudaDataType_t in_t = p.bf16 ? CUDA_R_16BF : CUDA_R_32F;
    const size_t esz = p.bf16 ? 2 : 4;
    for (int64_t b = 0; b < d.batch; ++b)
        F5_TRY(blas_check(cublasGemmStridedBatchedEx(p.blas, CUBLAS_OP_T, CUBLAS_OP_N, int(cig), int(T), int(J), &one, wr, in_t, int(J),
                                                     int64_t(cig) * J, reinterpret_cast<const char *>(p.col) + size_t(b) * G * T * J * esz,
                                                     in_t, int(J), int64_t(T) * J, &zero, dst + size_t(b) * T * D, CUDA_R_32F, int(D),
                                                     int64_t(cig), kPosGroups, p.bf16 ? CUBLAS_COMPUTE_32F : p.compute,
                                                     CUBLAS_GEMM_DEFAULT),
                          "position convolution"));
    return VOX_CUDA_OK;
}

// The input embedding into p.h: [x | cond] . W_in^T + b as two accumulating GEMMs over the two column blocks of W_in,
// then h += mish(conv2(mish(conv1(h) + b1)) + b2).
int record_embed(F5Plan &p, cudaStream_t st) {
    const vox_cuda_f5_desc &d = p.d;
    const int64_t R = p.R, D = d.dim, M = d.out_dim, C = d.in_dim - d.out_dim;
    const float one = 1.0f, zero = 0.0f;
    if (p.tc && (p.tc_mask & 32)) {  // [x | cond] in bf16, then one GEMM with the bias in its epilogue
        const uint32_t ne = uint32_t(R * (M + C));
        launch_k(f5_concat_bf16_kernel, grid_for(ne, 256, 4), 256, 0, st, (const float *)p.xin, (const float *)p.cond, p.xc_b, ne,
                 uint32_t(M), uint32_t(C));
        F5_TRY(check_launch("vox_cuda_f5 in_proj input"));
        F5_TRY(gemm_run(p.g_in, st, "vox_cuda_f5 in_proj"));
    } else {
        F5_TRY(blas_check(cublasGemmEx(p.blas, CUBLAS_OP_T, CUBLAS_OP_N, int(D), int(R), int(M), &one, d.in_proj, CUDA_R_32F, d.in_dim,
                                       p.xin, CUDA_R_32F, int(M), &zero, p.h, CUDA_R_32F, int(D), p.compute, CUBLAS_GEMM_DEFAULT),
                          "in_proj (x)"));
        F5_TRY(blas_check(cublasGemmEx(p.blas, CUBLAS_OP_T, CUBLAS_OP_N, int(D), int(R), int(C), &one, d.in_proj + M, CUDA_R_32F, d.in_dim,
                                       p.cond, CUDA_R_32F, int(C), &one, p.h, CUDA_R_32F, int(D), p.compute, CUBLAS_GEMM_DEFAULT),
                          "in_proj (cond)"));
        if (d.in_proj_b) F5_TRY(vox_cuda_bias_add(p.h, d.in_proj_b, R, D, VOX_CUDA_F32, st));
    }
    const uint32_t n = uint32_t(R * D);
    F5_TRY(conv_pos(p, p.h, p.w1r, p.ctmp, p.tc && (p.tc_mask & 32) ? &p.g_conv1 : nullptr, st));
    launch_k(f5_bias_mish_kernel, grid_for(n, 256, 4), 256, 0, st, p.ctmp, d.pos1_b, (float *)nullptr, n, uint32_t(D));
    F5_TRY(check_launch("vox_cuda_f5 mish"));
    F5_TRY(conv_pos(p, p.ctmp, p.w2r, p.o, p.tc && (p.tc_mask & 32) ? &p.g_conv2 : nullptr, st));
    launch_k(f5_bias_mish_kernel, grid_for(n, 256, 4), 256, 0, st, p.o, d.pos2_b, p.h, n, uint32_t(D));
    return check_launch("vox_cuda_f5 mish");
}

// The whole step on stream st, f32 / TF32 path (eager or under capture; cuBLAS is bound to the same stream).
int record(F5Plan &p, cudaStream_t st) {
    const vox_cuda_f5_desc &d = p.d;
    const int64_t R = p.R, D = d.dim, IN = p.inner, FF = p.ff;
    if (p.embed) F5_TRY(record_embed(p, st));
    const uint32_t rope_heads = uint32_t(d.pe_attn_head > 0 ? d.pe_attn_head : d.heads);
    const uint32_t half = uint32_t(d.dim_head / 2);
    const uint32_t pairs = uint32_t(R) * rope_heads * half;
    const int rope_grid = grid_for(pairs, 256, 4);
    auto bias = [&](float *y, const float *b, int64_t rows, int64_t cols) {
        return b ? vox_cuda_bias_add(y, b, rows, cols, VOX_CUDA_F32, st) : VOX_CUDA_OK;
    };
    for (const vox_cuda_f5_block_weights &L : p.blocks) {
        F5_TRY(gemm_xwt(p, p.ts, L.ada, p.ada, 1, 6 * D, D));
        F5_TRY(bias(p.ada, L.ada_b, 1, 6 * D));
        const float *shift_msa = p.ada, *scale_msa = p.ada + D, *gate_msa = p.ada + 2 * D;
        const float *shift_mlp = p.ada + 3 * D, *scale_mlp = p.ada + 4 * D, *gate_mlp = p.ada + 5 * D;
        F5_TRY(vox_cuda_adaln(p.h, shift_msa, scale_msa, nullptr, nullptr, p.nrm, 1, R, D, 1e-6f, VOX_CUDA_F32, st));
        F5_TRY(gemm_xwt(p, p.nrm, L.q, p.q, R, IN, D));
        F5_TRY(gemm_xwt(p, p.nrm, L.k, p.k, R, IN, D));
        F5_TRY(gemm_xwt(p, p.nrm, L.v, p.v, R, IN, D));
        F5_TRY(bias(p.q, L.q_b, R, IN));
        F5_TRY(bias(p.k, L.k_b, R, IN));
        F5_TRY(bias(p.v, L.v_b, R, IN));
        launch_k(f5_rope_kernel, rope_grid, 256, 0, st, p.q, p.k, (const float2 *)p.cs, pairs, uint32_t(d.frames), half, rope_heads,
                 uint32_t(d.dim_head), uint32_t(IN));
        F5_TRY(check_launch("vox_cuda_f5 rope"));
        for (int64_t b = 0; b < d.batch; ++b) F5_TRY(attention(p, b, st));
        F5_TRY(gemm_xwt(p, p.at, L.o, p.o, R, D, IN));
        F5_TRY(bias(p.o, L.o_b, R, D));
        F5_TRY(vox_cuda_gated_add(p.h, gate_msa, p.o, 1, R, D, VOX_CUDA_F32, st));
        F5_TRY(vox_cuda_adaln(p.h, shift_mlp, scale_mlp, nullptr, nullptr, p.nrm, 1, R, D, 1e-6f, VOX_CUDA_F32, st));
        F5_TRY(gemm_xwt(p, p.nrm, L.ff1, p.ffb, R, FF, D));
        F5_TRY(bias(p.ffb, L.ff1_b, R, FF));
        F5_TRY(vox_cuda_gelu(p.ffb, p.ffb, R * FF, VOX_CUDA_GELU_TANH, VOX_CUDA_F32, st));
        F5_TRY(gemm_xwt(p, p.ffb, L.ff2, p.o, R, D, FF));
        F5_TRY(bias(p.o, L.ff2_b, R, D));
        F5_TRY(vox_cuda_gated_add(p.h, gate_mlp, p.o, 1, R, D, VOX_CUDA_F32, st));
    }
    F5_TRY(gemm_xwt(p, p.ts, d.norm_out, p.fin, 1, 2 * D, D));  // fin = [scale, shift] (f5.cpp:720-722)
    F5_TRY(bias(p.fin, d.norm_out_b, 1, 2 * D));
    F5_TRY(vox_cuda_adaln(p.h, p.fin + D, p.fin, nullptr, nullptr, p.nrm, 1, R, D, 1e-6f, VOX_CUDA_F32, st));
    F5_TRY(gemm_xwt(p, p.nrm, d.proj_out, p.out, R, d.out_dim, D));
    return bias(p.out, d.proj_out_b, R, d.out_dim);
}

// h += gate * delta (if delta), then nrm_b = modulated LayerNorm of h in bf16.
int resmod(F5Plan &p, const float *delta, const float *dbias, const float *gate, const float *scale, const float *shift,
           cudaStream_t st) {
    const uint32_t R = uint32_t(p.R), D = uint32_t(p.d.dim), vpl = (D / 4 + 31) / 32;
    uint2 *nrm = reinterpret_cast<uint2 *>(p.nrm_b);
    if (vpl >= 8) {  // four warps a row: four times the rows' loads in flight for the step's 2 x 1024 rows
        const int g = int((4 * R + 7) / 8);
        if (vpl <= 8) launch_k(f5_resmod_kernel<2, 4>, g, 256, 0, st, p.h, delta, dbias, gate, scale, shift, nrm, R, D, 1e-6f);
        else launch_k(f5_resmod_kernel<4, 4>, g, 256, 0, st, p.h, delta, dbias, gate, scale, shift, nrm, R, D, 1e-6f);
        return check_launch("vox_cuda_f5 residual/modulate");
    }
    const int g = int((R + 7) / 8);
    if (vpl <= 1) launch_k(f5_resmod_kernel<1, 1>, g, 256, 0, st, p.h, delta, dbias, gate, scale, shift, nrm, R, D, 1e-6f);
    else if (vpl <= 2) launch_k(f5_resmod_kernel<2, 1>, g, 256, 0, st, p.h, delta, dbias, gate, scale, shift, nrm, R, D, 1e-6f);
    else if (vpl <= 4) launch_k(f5_resmod_kernel<4, 1>, g, 256, 0, st, p.h, delta, dbias, gate, scale, shift, nrm, R, D, 1e-6f);
    else if (vpl <= 8) launch_k(f5_resmod_kernel<8, 1>, g, 256, 0, st, p.h, delta, dbias, gate, scale, shift, nrm, R, D, 1e-6f);
    else launch_k(f5_resmod_kernel<16, 1>, g, 256, 0, st, p.h, delta, dbias, gate, scale, shift, nrm, R, D, 1e-6f);
    return check_launch("vox_cuda_f5 residual/modulate");
}

// The whole step, bf16 path: the same arithmetic with bf16 GEMM inputs, the residual stream h in f32, each block's
// closing gated residual fused with the next modulation.
int record_bf16(F5Plan &p, cudaStream_t st) {
    const vox_cuda_f5_desc &d = p.d;
    const int64_t R = p.R, D = d.dim, IN = p.inner, FF = p.ff, L = d.depth;
    if (p.embed) F5_TRY(record_embed(p, st));
    // every block's ada vectors (f32 weights, bias added), then fin = [scale, shift] (f5.cpp:720-722)
    const float *const *wt = reinterpret_cast<const float *const *>(p.ada_ptrs);
    launch_k(f5_gemv_f32_kernel, dim3(unsigned((6 * D + 7) / 8), unsigned(L)), 256, 0, st, wt, (const float *)p.ts, (const float *)p.b_ada,
             p.ada_all, uint32_t(6 * D), uint32_t(D));
    F5_TRY(check_launch("vox_cuda_f5 ada"));
    launch_k(f5_gemv_f32_kernel, dim3(unsigned((2 * D + 7) / 8), 1u), 256, 0, st, wt + 3 * L, (const float *)p.ts, (const float *)p.b_fin,
             p.fin, uint32_t(2 * D), uint32_t(D));
    F5_TRY(check_launch("vox_cuda_f5 norm_out"));
    const uint32_t rope_heads = uint32_t(d.pe_attn_head > 0 ? d.pe_attn_head : d.heads);
    const uint32_t qkv_octs = uint32_t(R * 3 * IN / 8), ff_octs = uint32_t(R * FF / 8);
    const dim3 fgt(unsigned((d.frames + kTcRows - 1) / kTcRows), unsigned(d.heads), unsigned(d.batch));
    // two threads a query row (VOX_CUDA_F5_ATTN=1: one thread a row, for comparisons)
    const char *eattn = std::getenv("VOX_CUDA_F5_ATTN");
    const bool attn1 = eattn && eattn[0] == '1';
    if (cudaFuncSetAttribute(f5_flash_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTcSmem)) != cudaSuccess ||
        cudaFuncSetAttribute(f5_flash_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTc2Smem)) != cudaSuccess)
        return check_launch("vox_cuda_f5 attention (shared memory)");
    const float scale_log2 = float(1.4426950408889634 / std::sqrt(double(d.dim_head)));
    F5_TRY(resmod(p, nullptr, nullptr, nullptr, p.ada_all + D, p.ada_all, st));
    for (int64_t l = 0; l < L; ++l) {
        const float *A = p.ada_all + l * 6 * D;  // shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp
        if (p.tc && (p.tc_mask & 1)) {  // bias and RoPE in the GEMM's epilogue
            F5_TRY(gemm_run(p.g_qkv[size_t(l)], st, "vox_cuda_f5 q|k|v"));
        } else {
            F5_TRY(gemm_bf16(p, p.nrm_b, p.w_qkv + size_t(l) * 3 * IN * D, p.qkv_b, CUDA_R_16BF, R, 3 * IN, D));
            launch_k(f5_qkv_bias_rope_kernel, grid_for(qkv_octs, 256, 4), 256, 0, st, reinterpret_cast<uint4 *>(p.qkv_b),
                     (const float *)(p.b_qkv + size_t(l) * 3 * IN), (const float2 *)p.cs, qkv_octs, uint32_t(d.frames),
                     uint32_t(d.dim_head / 2), rope_heads, uint32_t(d.dim_head), uint32_t(IN));
            F5_TRY(check_launch("vox_cuda_f5 bias/rope (bf16)"));
        }
        if (attn1)
            launch_k(f5_flash_tc_kernel, fgt, kTcThreads, kTcSmem, st, (const __nv_bfloat16 *)p.qkv_b, (const __nv_bfloat16 *)(p.qkv_b + IN),
                     (const __nv_bfloat16 *)(p.qkv_b + 2 * IN), (__nv_bfloat16 *)p.at_b, int(d.frames), int(3 * IN), int(IN), scale_log2);
        else
            launch_k(f5_flash_tc2_kernel, fgt, kTc2Threads, kTc2Smem, st, (const __nv_bfloat16 *)p.qkv_b, (const __nv_bfloat16 *)(p.qkv_b + IN),
                     (const __nv_bfloat16 *)(p.qkv_b + 2 * IN), (__nv_bfloat16 *)p.at_b, int(d.frames), int(3 * IN), int(IN), scale_log2);
        F5_TRY(check_launch("vox_cuda_f5 attention"));
        if (p.tc && (p.tc_mask & 2)) F5_TRY(gemm_run(p.g_o[size_t(l)], st, "vox_cuda_f5 o"));
        else F5_TRY(gemm_bf16(p, p.at_b, p.w_o + size_t(l) * D * IN, p.o, CUDA_R_32F, R, D, IN));
        F5_TRY(resmod(p, p.o, p.b_o + l * D, A + 2 * D, A + 4 * D, A + 3 * D, st));
        if (p.tc && (p.tc_mask & 4)) {  // bias and GELU-tanh in the ff1 GEMM's epilogue
            F5_TRY(gemm_run(p.g_ff1[size_t(l)], st, "vox_cuda_f5 ff1"));
        } else {
            F5_TRY(gemm_bf16(p, p.nrm_b, p.w_ff1 + size_t(l) * FF * D, p.ff_b, CUDA_R_16BF, R, FF, D));
            launch_k(f5_bias_gelu_kernel, grid_for(ff_octs, 256, 4), 256, 0, st, reinterpret_cast<uint4 *>(p.ff_b),
                     (const float *)(p.b_ff1 + l * FF), ff_octs, uint32_t(FF));
            F5_TRY(check_launch("vox_cuda_f5 bias/gelu (bf16)"));
        }
        if (p.tc && (p.tc_mask & 8)) F5_TRY(gemm_run(p.g_ff2[size_t(l)], st, "vox_cuda_f5 ff2"));
        else F5_TRY(gemm_bf16(p, p.ff_b, p.w_ff2 + size_t(l) * D * FF, p.o, CUDA_R_32F, R, D, FF));
        if (l + 1 < L) {
            const float *An = A + 6 * D;
            F5_TRY(resmod(p, p.o, p.b_ff2 + l * D, A + 5 * D, An + D, An, st));
        } else {
            F5_TRY(resmod(p, p.o, p.b_ff2 + l * D, A + 5 * D, p.fin, p.fin + D, st));
        }
    }
    if (p.tc && (p.tc_mask & 16)) return gemm_run(p.g_proj, st, "vox_cuda_f5 proj_out");
    F5_TRY(gemm_bf16(p, p.nrm_b, p.w_proj, p.out, CUDA_R_32F, R, d.out_dim, D));
    return vox_cuda_bias_add(p.out, p.b_proj, R, d.out_dim, VOX_CUDA_F32, st);
}

void release(F5Plan *p) {
    if (!p) return;
    if (p->cap) cudaStreamSynchronize(p->cap);
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    if (p->blas) cublasDestroy(p->blas);
    for (void *b : {(void *)p->ws, (void *)p->h, (void *)p->ts, (void *)p->out, (void *)p->nrm, (void *)p->q, (void *)p->k,
                    (void *)p->v, (void *)p->at, (void *)p->o, (void *)p->ffb, (void *)p->s, (void *)p->ada, (void *)p->fin,
                    (void *)p->cs, (void *)p->qkv_b, (void *)p->ada_all, (void *)p->nrm_b, (void *)p->at_b, (void *)p->ff_b, (void *)p->w_qkv, (void *)p->w_o, (void *)p->w_ff1,
                    (void *)p->w_ff2, (void *)p->w_proj, (void *)p->ada_ptrs, (void *)p->b_ada, (void *)p->b_qkv, (void *)p->b_o,
                    (void *)p->b_ff1, (void *)p->b_ff2, (void *)p->b_fin, (void *)p->b_proj, (void *)p->xin, (void *)p->cond,
                    (void *)p->col, (void *)p->ctmp, (void *)p->w1r, (void *)p->w2r, (void *)p->xc_b, (void *)p->w_in})
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

// dst[0 .. n) = bf16(src) on stream st (n even).
int to_bf16(const float *src, __nv_bfloat16 *dst, size_t n, cudaStream_t st) {
    launch_k(f5_to_bf16_kernel, grid_for(int64_t(n / 2), 256, 4), 256, 0, st, reinterpret_cast<const float2 *>(src),
             reinterpret_cast<uint32_t *>(dst), n / 2);
    return check_launch("vox_cuda_f5_create (weights to bf16)");
}

// The tcgen05 GEMMs of the bf16 step, on the plan's own buffers (their tensor maps encode those addresses).
int build_gemms(F5Plan &p) {
    const vox_cuda_f5_desc &d = p.d;
    const int R = int(p.R), D = d.dim, IN = int(p.inner), FF = int(p.ff), L = d.depth;
    const char *nm = "vox_cuda_f5_create (GEMMs)";
    // VOX_CUDA_F5_TILES="qkv=1192,o=128,ff1=256,ff2=128" fixes a projection's tile (1000 * pair + columns; for
    // comparisons), else gemm_plan chooses
    const char *et = std::getenv("VOX_CUDA_F5_TILES");
    auto tile_of = [&](const char *key) {
        if (!et) return 0;
        const std::string t(et), k = std::string(key) + "=";
        size_t i = t.find(k);
        while (i != std::string::npos && i > 0 && t[i - 1] != ',') i = t.find(k, i + 1);
        return i == std::string::npos ? 0 : std::atoi(t.c_str() + i + k.size());
    };
    auto plan = [&](const void *x, int64_t ldx, const void *w, int64_t ldw, int N, int K, void *y, int64_t ldy, const float *bias, int epi,
                    GemmPlan &gp) {
        GemmArgs a;
        a.M = R, a.N = N, a.K = K, a.y = y, a.ldy = ldy, a.bias = bias;
        a.tile = tile_of(epi == kEpiQkvRope ? "qkv" : epi == kEpiGeluTanh ? "ff1" : y == p.o && K == FF ? "ff2" : y == p.o ? "o" : "other");
        // the fused q|k|v projection on 128 x 256 tiles: in the step it measured faster than the shape gemm_plan picks
        // alone (256 x 192 pairs; 2.213 against 2.238 ms a step, same box), its RoPE epilogue being the difference
        if (epi == kEpiQkvRope && !a.tile && N % 256 == 0) a.tile = 256;
        a.w_early = 1;  // the plan's bf16 weight snapshots: no kernel of the step writes them
        if (epi == kEpiQkvRope) {
            a.cs = p.cs, a.frames = d.frames, a.rope_heads = d.pe_attn_head > 0 ? d.pe_attn_head : d.heads, a.hd = d.dim_head, a.inner = IN;
        }
        return gemm_plan(x, ldx, w, ldw, a, epi, gp, nm);
    };
    p.g_qkv.resize(size_t(L)), p.g_o.resize(size_t(L)), p.g_ff1.resize(size_t(L)), p.g_ff2.resize(size_t(L));
    for (int l = 0; l < L; ++l) {
        const size_t ls = size_t(l);
        F5_TRY(plan(p.nrm_b, D, p.w_qkv + ls * 3 * IN * D, D, 3 * IN, D, p.qkv_b, 3 * IN, p.b_qkv + ls * 3 * IN, kEpiQkvRope, p.g_qkv[ls]));
        F5_TRY(plan(p.at_b, IN, p.w_o + ls * D * IN, IN, D, IN, p.o, D, nullptr, kEpiF32, p.g_o[ls]));
        F5_TRY(plan(p.nrm_b, D, p.w_ff1 + ls * FF * D, D, FF, D, p.ff_b, FF, p.b_ff1 + ls * FF, kEpiGeluTanh, p.g_ff1[ls]));
        F5_TRY(plan(p.ff_b, FF, p.w_ff2 + ls * D * FF, FF, D, FF, p.o, D, nullptr, kEpiF32, p.g_ff2[ls]));
    }
    F5_TRY(plan(p.nrm_b, D, p.w_proj, D, d.out_dim, D, p.out, d.out_dim, p.b_proj, kEpiF32, p.g_proj));
    if (p.embed) {
        F5_TRY(plan(p.xc_b, d.in_dim, p.w_in, d.in_dim, D, d.in_dim, p.h, D, d.in_proj_b, kEpiF32, p.g_in));
        // position convolutions: x planes [batch][group] of the im2col [T][J], W planes [group][cig][J], y columns g cig
        const int cig = D / kPosGroups, J = kPosK * cig;
        const void *wrs[2] = {p.w1r, p.w2r};
        float *dsts[2] = {p.ctmp, p.o};
        GemmPlan *gps[2] = {&p.g_conv1, &p.g_conv2};
        for (int i = 0; i < 2; ++i) {
            GemmArgs a;
            a.M = d.frames, a.N = cig, a.K = J, a.batches = d.batch, a.groups = kPosGroups;
            a.y = dsts[i], a.ldy = D, a.y_bstride = int64_t(d.frames) * D, a.y_gstride = cig;
            F5_TRY(gemm_plan(p.col, J, wrs[i], J, a, kEpiF32, *gps[i], nm));
        }
    }
    return VOX_CUDA_OK;
}

int build(F5Plan &p, cudaStream_t user) {
    const vox_cuda_f5_desc &d = p.d;
    const size_t R = size_t(p.R), D = size_t(d.dim), IN = size_t(p.inner), FF = size_t(p.ff), N = size_t(d.frames), L = size_t(d.depth);
    p.bf16 = d.math == VOX_CUDA_F5_MATH_BF16 && d.dim_head == kFaHd && D % 4 == 0 && D <= 2048 && FF % 8 == 0;
    F5_TRY(alloc(&p.h, R * D, "h"));
    F5_TRY(alloc(&p.ts, D, "ts"));
    F5_TRY(alloc(&p.out, R * size_t(d.out_dim), "out"));
    F5_TRY(alloc(&p.o, R * D, "o"));
    F5_TRY(alloc(&p.fin, 2 * D, "fin"));
    F5_TRY(alloc(&p.cs, N * size_t(d.dim_head / 2), "rope table"));
    p.embed = d.in_proj != nullptr;
    {
        const int64_t cig = d.dim / kPosGroups;
        // VOX_CUDA_F5_GEMM=cublas keeps the bf16 step's GEMMs on cuBLAS; VOX_CUDA_F5_TC_MASK (bits: 1 q|k|v, 2 o, 4 ff1,
        // 8 ff2, 16 proj_out, 32 input embedding) picks the ones on this library's kernel (for comparisons)
        const char *e = std::getenv("VOX_CUDA_F5_GEMM");
        const bool cublas = e && std::string(e) == "cublas";
        const char *mk = std::getenv("VOX_CUDA_F5_TC_MASK");
        p.tc_mask = mk ? std::atoi(mk) : 63;
        p.tc = !cublas && p.bf16 && D % 8 == 0 && IN % 32 == 0 && FF % 8 == 0 && d.dim_head % 32 == 0 &&
               (!p.embed || (d.in_dim % 8 == 0 && d.dim % kPosGroups == 0 && cig % 8 == 0));
    }
    if (p.bf16) {
        F5_TRY(alloc(&p.qkv_b, R * 3 * IN, "q|k|v (bf16)"));
        F5_TRY(alloc(&p.ada_all, L * 6 * D, "ada"));
        F5_TRY(alloc(&p.nrm_b, R * D, "nrm (bf16)"));
        F5_TRY(alloc(&p.at_b, R * IN, "attention (bf16)"));
        F5_TRY(alloc(&p.ff_b, R * FF, "ff (bf16)"));
        F5_TRY(alloc(&p.w_qkv, L * 3 * IN * D, "q|k|v weights (bf16)"));
        F5_TRY(alloc(&p.w_o, L * D * IN, "o weights (bf16)"));
        F5_TRY(alloc(&p.w_ff1, L * FF * D, "ff1 weights (bf16)"));
        F5_TRY(alloc(&p.w_ff2, L * D * FF, "ff2 weights (bf16)"));
        F5_TRY(alloc(&p.w_proj, size_t(d.out_dim) * D, "proj_out weights (bf16)"));
        F5_TRY(alloc(&p.ada_ptrs, 3 * L + 1, "ada pointers"));
        for (size_t l = 0; l < L; ++l) {
            const vox_cuda_f5_block_weights &B = p.blocks[l];
            F5_TRY(to_bf16(B.q, p.w_qkv + l * 3 * IN * D, IN * D, user));
            F5_TRY(to_bf16(B.k, p.w_qkv + l * 3 * IN * D + IN * D, IN * D, user));
            F5_TRY(to_bf16(B.v, p.w_qkv + l * 3 * IN * D + 2 * IN * D, IN * D, user));
            F5_TRY(to_bf16(B.o, p.w_o + l * D * IN, D * IN, user));
            F5_TRY(to_bf16(B.ff1, p.w_ff1 + l * FF * D, FF * D, user));
            F5_TRY(to_bf16(B.ff2, p.w_ff2 + l * D * FF, D * FF, user));
        }
        F5_TRY(to_bf16(d.proj_out, p.w_proj, size_t(d.out_dim) * D, user));
        F5_TRY(alloc(&p.b_ada, L * 6 * D, "ada biases"));
        F5_TRY(alloc(&p.b_qkv, L * 3 * IN, "q|k|v biases"));
        F5_TRY(alloc(&p.b_o, L * D, "o biases"));
        F5_TRY(alloc(&p.b_ff1, L * FF, "ff1 biases"));
        F5_TRY(alloc(&p.b_ff2, L * D, "ff2 biases"));
        F5_TRY(alloc(&p.b_fin, 2 * D, "norm_out bias"));
        F5_TRY(alloc(&p.b_proj, size_t(d.out_dim), "proj_out bias"));
        auto snap = [&](float *dst, const float *src, size_t n) {  // the bias, or zeros
            const cudaError_t e = src ? cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, user) : cudaMemsetAsync(dst, 0, n * 4, user);
            return e == cudaSuccess ? VOX_CUDA_OK : check_launch("vox_cuda_f5_create (biases)");
        };
        for (size_t l = 0; l < L; ++l) {
            const vox_cuda_f5_block_weights &B = p.blocks[l];
            F5_TRY(snap(p.b_ada + l * 6 * D, B.ada_b, 6 * D));
            F5_TRY(snap(p.b_qkv + l * 3 * IN, B.q_b, IN));
            F5_TRY(snap(p.b_qkv + l * 3 * IN + IN, B.k_b, IN));
            F5_TRY(snap(p.b_qkv + l * 3 * IN + 2 * IN, B.v_b, IN));
            F5_TRY(snap(p.b_o + l * D, B.o_b, D));
            F5_TRY(snap(p.b_ff1 + l * FF, B.ff1_b, FF));
            F5_TRY(snap(p.b_ff2 + l * D, B.ff2_b, D));
        }
        F5_TRY(snap(p.b_fin, d.norm_out_b, 2 * D));
        F5_TRY(snap(p.b_proj, d.proj_out_b, size_t(d.out_dim)));
        std::vector<const void *> ptrs(3 * L + 1);
        for (size_t l = 0; l < L; ++l) {
            ptrs[l] = p.blocks[l].ada;
            ptrs[L + l] = p.ts;
            ptrs[2 * L + l] = p.ada_all + l * 6 * D;
        }
        ptrs[3 * L] = d.norm_out;
        if (cudaMemcpy(p.ada_ptrs, ptrs.data(), ptrs.size() * sizeof(void *), cudaMemcpyHostToDevice) != cudaSuccess)
            return check_launch("vox_cuda_f5_create");
    } else {
        F5_TRY(alloc(&p.nrm, R * D, "nrm"));
        F5_TRY(alloc(&p.q, R * IN, "q"));
        F5_TRY(alloc(&p.k, R * IN, "k"));
        F5_TRY(alloc(&p.v, R * IN, "v"));
        F5_TRY(alloc(&p.at, R * IN, "at"));
        F5_TRY(alloc(&p.ffb, R * FF, "ff"));
        F5_TRY(alloc(&p.s, size_t(d.heads) * N * N, "scores"));
        F5_TRY(alloc(&p.ada, 6 * D, "ada"));
    }
    if (p.embed) {
        const size_t cig = D / kPosGroups, J = size_t(kPosK) * cig, nw = D * J;
        if (p.tc) {
            F5_TRY(alloc(&p.xc_b, R * size_t(d.in_dim), "in_proj input (bf16)"));
            F5_TRY(alloc(&p.w_in, D * size_t(d.in_dim), "in_proj weights (bf16)"));
            F5_TRY(to_bf16(d.in_proj, p.w_in, D * size_t(d.in_dim), user));
        }
        F5_TRY(alloc(&p.xin, R * size_t(d.out_dim), "x"));
        F5_TRY(alloc(&p.cond, R * size_t(d.in_dim - d.out_dim), "cond"));
        F5_TRY(alloc(&p.col, size_t(d.batch) * kPosGroups * N * J, "im2col"));
        F5_TRY(alloc(&p.ctmp, R * D, "convolution"));
        F5_TRY(alloc(&p.w1r, nw, "conv1 weights"));
        F5_TRY(alloc(&p.w2r, nw, "conv2 weights"));
        if (cudaMemsetAsync(p.xin, 0, R * size_t(d.out_dim) * 4, user) != cudaSuccess ||
            cudaMemsetAsync(p.cond, 0, R * size_t(d.in_dim - d.out_dim) * 4, user) != cudaSuccess)
            return check_launch("vox_cuda_f5_create");
        for (auto [w, wr] : {std::make_pair(d.pos1_w, p.w1r), std::make_pair(d.pos2_w, p.w2r)}) {
            if (p.bf16)
                launch_k(f5_conv_reorder_kernel<__nv_bfloat16>, grid_for(int64_t(nw), 256, 4), 256, 0, user, w,
                         reinterpret_cast<__nv_bfloat16 *>(wr), uint32_t(nw), uint32_t(cig), uint32_t(kPosK));
            else
                launch_k(f5_conv_reorder_kernel<float>, grid_for(int64_t(nw), 256, 4), 256, 0, user, w, wr, uint32_t(nw), uint32_t(cig),
                         uint32_t(kPosK));
            F5_TRY(check_launch("vox_cuda_f5_create (conv weights)"));
        }
    }
    if (p.tc) F5_TRY(build_gemms(p));
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
    if (cudaStreamCreateWithFlags(&p.cap, cudaStreamNonBlocking) != cudaSuccess) return check_launch("vox_cuda_f5_create");
    if (!p.tc || p.tc_mask != 63) {  // cuBLAS only where a GEMM of the step is not on this library's tcgen05 kernel
        F5_TRY(alloc(reinterpret_cast<uint8_t **>(&p.ws), kBlasWorkspace, "cuBLAS workspace"));
        F5_TRY(blas_check(cublasCreate(&p.blas), "create"));
        F5_TRY(blas_check(cublasSetMathMode(p.blas, d.math == VOX_CUDA_F5_MATH_F32 ? CUBLAS_PEDANTIC_MATH : CUBLAS_DEFAULT_MATH), "math mode"));
        p.compute = d.math == VOX_CUDA_F5_MATH_TF32   ? CUBLAS_COMPUTE_32F_FAST_TF32
                    : d.math == VOX_CUDA_F5_MATH_BF16 ? CUBLAS_COMPUTE_32F_FAST_16BF
                                                      : CUBLAS_COMPUTE_32F_PEDANTIC;
        // stream and workspace set once, outside the capture (no cuBLAS allocation may happen while capturing)
        F5_TRY(blas_check(cublasSetStream(p.blas, p.cap), "set stream"));
        F5_TRY(blas_check(cublasSetWorkspace(p.blas, p.ws, kBlasWorkspace), "set workspace"));
    }
    // the capture stream starts after the caller's work so far (weight conversion, the table, the zeroed inputs)
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return check_launch("vox_cuda_f5_create");
    cudaEventRecord(ev, user);
    cudaStreamWaitEvent(p.cap, ev, 0);
    cudaEventDestroy(ev);
    auto rec = [&p](cudaStream_t st) { return p.bf16 ? record_bf16(p, st) : record(p, st); };
    F5_TRY(rec(p.cap));  // eager run: algorithm selection and first-use kernel attributes outside the capture
    if (cudaStreamSynchronize(p.cap) != cudaSuccess) return check_launch("vox_cuda_f5_create (eager run)");
    if (cudaStreamBeginCapture(p.cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return check_launch("vox_cuda_f5_create (capture)");
    const int rc = rec(p.cap);
    const cudaError_t end = cudaStreamEndCapture(p.cap, &p.graph);
    if (rc != VOX_CUDA_OK) return rc;
    if (end != cudaSuccess) return check_launch("vox_cuda_f5_create (end capture)");
    if (cudaGraphInstantiate(&p.exec, p.graph, 0) != cudaSuccess) return check_launch("vox_cuda_f5_create (instantiate)");
    return VOX_CUDA_OK;
}

}  // namespace

int f5_take_device_error(unsigned int *flags) { return take_device_error(flags); }

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
    VOX_REQUIRE(!d.in_proj || (d.in_dim > d.out_dim && d.pos1_w && d.pos2_w && d.dim % kPosGroups == 0 &&
                               int64_t(d.batch) * kPosGroups * d.frames * kPosK * (d.dim / kPosGroups) < (int64_t(1) << 32)),
                "vox_cuda_f5_create: the input embedding needs in_dim > out_dim, both convolutions and dim % 16 == 0");
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

int vox_cuda_f5_inputs(vox_cuda_f5 *plan, float **x, float **cond) {
    VOX_REQUIRE(plan, "vox_cuda_f5_inputs: NULL plan");
    F5Plan *p = reinterpret_cast<F5Plan *>(plan);
    if (x) *x = p->xin;
    if (cond) *cond = p->cond;
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
