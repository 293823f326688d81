// Quantized matrix-vector product for decoding: y[i][r] = bias[r] + sum_k W[r][k] x[i][k] (or y += ...) for up to
// 8 activation rows per launch, W in Vox's Q8 (int8 + one scale per 32 weights) or Q4 (4-bit, 16 bytes per
// 32-block) layout, x and y f32 — the semantics of Vox's GPU matvec (shaders/matmul.comp:1-8, dispatched for
// m <= 8 by rec_mm, gpu_vulkan.cpp:657-674) and of the CPU matmul's dequantise-then-f32 path (kernels.cpp:669-688).
//
// The product runs on the tensor cores with f32 accuracy. Every weight code is an integer that bf16 represents
// exactly (Q8: -128..127, Q4: -8..7), converted in registers; each activation is split into three bf16 parts
// x = x1 + x2 + x3 (24 significant bits), so every product code * part is exact in the f32 accumulator of
// mma.sync.m16n8k16 (bf16 in, f32 accumulate) and the result carries the rounding of an f32 dot product. The eight
// activation rows are the MMA's N = 8 columns; the weight rows its M. The 32-weight block scale multiplies the
// block's partial product (6 MMAs: two k16 steps x three parts) in f32. Weights go from registers straight into the
// MMA: tcgen05 would need them staged through shared memory (4 bytes of shared traffic per weight at HBM rate).
//
// Work split: a CTA (8 warps) owns 256 weight rows (32 per warp: two 16-row MMA tiles) and one K slice; the C CTAs
// of a thread-block cluster cover the same rows and consecutive K slices. Each warp streams its 32 rows' weights
// through its own shared-memory ring: one 1-D bulk copy (TMA) per row per chunk of kChunk blocks, completed on the
// stage's mbarrier, kStages chunks in flight, so the bytes in flight cost no registers. Meanwhile the CTA writes its
// slice's activation splits into shared memory in B-fragment order (each split computed once per CTA, read by every
// warp with three 16-byte loads per block) and stages its block scales there. The C partial sums are added in fixed
// rank order through distributed shared memory: deterministic, no scratch.
//
// Within one MMA the k index is permuted the same way for both operands (thread t of a row quad takes 8
// consecutive weights of the block: a dot product does not depend on the order of its terms).
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "rows.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace voxcuda {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTiles = 1;                 // 16-row MMA tiles per warp
constexpr int kWarpRows = 16 * kTiles;    // 16
constexpr int kRows = kWarps * kWarpRows; // weight rows per CTA (128)
constexpr int kTok = 8;                   // activation rows per launch (the MMA's N)
constexpr int kRedPad = kRows + 4;        // row stride of the reduction buffer (conflict-free fragment stores)
constexpr int kStages = 3;                // weight chunks in flight per warp
constexpr int kMaxCluster = 16;
constexpr int kChunkBytes = 128;          // bytes of every row per staged chunk (Q8: 4 blocks, Q4: 8)
template <bool Q4> __host__ __device__ constexpr int chunk_blocks() { return Q4 ? kChunkBytes / 16 : kChunkBytes / 32; }

struct GemvArgs {
    const uint8_t *w;
    const void *scale;
    const float *bias;
    const float *x;   // [m][cols], m <= 8
    float *y;         // [m][rows] (row stride ystride)
    int64_t rows, cols, ystride;
    int m, accumulate, nblk, bps;  // bps: 32-blocks per K slice (one slice per CTA of a cluster)
    FastDiv bdiv;                  // division by bps
};

// A staged chunk is the TMA box [32 rows][128 bytes] in the 128-byte swizzle: the 16-byte piece p of row r sits at
// r * 128 + ((p ^ (r % 8)) * 16), so the lanes' reads of the same piece of rows g = 0..7 hit 8 different 16-byte bank
// groups (no conflicts).
constexpr int kStageBytes = kWarpRows * kChunkBytes;  // 2 KB, 1024-byte aligned
template <bool Q4> __host__ __device__ constexpr int stage_bytes() { return kStageBytes; }
__device__ __forceinline__ int swz(int r, int off) { return r * kChunkBytes + ((((off >> 4) ^ r) & 7) << 4) + (off & 15); }

// Dynamic shared memory of a CTA: mbarriers [kWarps][kStages], weight rings [kWarps][kStages][stage] (after the main
// loop: the reduction buffer [kTok][kRedPad]), B fragments [bps][3 parts][4m lanes][4 words] (the lanes of the m
// activation rows; the others read zeros), scales [kRows][bps + 1] in their input type.
constexpr size_t kBarBytes = 1024;  // keeps the rings 1024-byte aligned (the swizzle's period)
template <bool Q4> __host__ __device__ constexpr size_t ring_bytes() { return size_t(kWarps) * kStages * stage_bytes<Q4>(); }
__host__ __device__ constexpr size_t frag_bytes(int bps, int m) { return size_t(bps) * 3 * 4 * m * 16; }
__host__ __device__ constexpr size_t scale_bytes(int bps, bool f16) { return (size_t(kRows) * (bps + 1) * (f16 ? 2 : 4) + 15) / 16 * 16; }
template <bool Q4> __host__ __device__ constexpr size_t gemv_smem(int bps, bool f16, int m) {
    return 1024 + kBarBytes + ring_bytes<Q4>() + frag_bytes(bps, m) + scale_bytes(bps, f16);  // + alignment slack
}
static_assert(size_t(kTok) * kRedPad * 4 <= ring_bytes<false>() && size_t(kTok) * kRedPad * 4 <= ring_bytes<true>(),
              "the reduction buffer reuses the weight rings");

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four int8 codes -> two bf16x2 words (codes 0,1 and 2,3), exact: 2^23 + (q + 128) is built in the f32 bit pattern
// and 2^23 + 128 subtracted; the integer's bf16 pattern is the high half of its f32 pattern (its low 16 bits are 0).
__device__ __forceinline__ void q8_to_bf16(uint32_t word, uint32_t &p01, uint32_t &p23) {
    const uint32_t u = word ^ 0x80808080u;
    const float2 m = make_float2(-8388736.0f, -8388736.0f);
    const float2 f01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                                              __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541))), m);
    const float2 f23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                                              __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543))), m);
    p01 = __byte_perm(__float_as_uint(f01.x), __float_as_uint(f01.y), 0x7632);
    p23 = __byte_perm(__float_as_uint(f23.x), __float_as_uint(f23.y), 0x7632);
}

// Four 4-bit codes (one per byte of nib, values 0..15) -> two bf16x2 words of code - 8, exact: the bf16 pattern
// 0x43nn is 128 + nn.
__device__ __forceinline__ void q4_to_bf16(uint32_t nib, uint32_t &p01, uint32_t &p23) {
    const __nv_bfloat162 off = __floats2bfloat162_rn(136.0f, 136.0f);
    uint32_t a = __byte_perm(nib, 0x43434343u, 0x5140), b = __byte_perm(nib, 0x43434343u, 0x5342);
    __nv_bfloat162 ra = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&a), off);
    __nv_bfloat162 rb = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&b), off);
    p01 = *reinterpret_cast<uint32_t *>(&ra);
    p23 = *reinterpret_cast<uint32_t *>(&rb);
}

// x = hi + mid + lo for two values, each part a bf16x2 word (the residuals are exact in f32).
__device__ __forceinline__ void split3(float a, float b, uint32_t &hi, uint32_t &mid, uint32_t &lo) {
    hi = bf16x2_rn(a, b);
    const float ar = a - __uint_as_float(hi << 16), br = b - __uint_as_float(hi & 0xFFFF0000u);
    mid = bf16x2_rn(ar, br);
    lo = bf16x2_rn(ar - __uint_as_float(mid << 16), br - __uint_as_float(mid & 0xFFFF0000u));
}

template <bool SF16>
__device__ __forceinline__ float load_scale(const void *s, int64_t i) {
    if (SF16) return __half2float(__ldg(reinterpret_cast<const __half *>(s) + i));
    return __ldg(reinterpret_cast<const float *>(s) + i);
}

// 2-D tensor copy (TMA) of the box at (x bytes, y rows) of `map` into this CTA's shared memory, completing on `bar`.
// The box lands in the issuing CTA only (no copy to other CTAs of the cluster).
__device__ __forceinline__ void tensor_g2s_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
                 : "memory");
}

// Position of weight k (0..31) of a block in the MMA operands: thread t of the row quad, k16 step j, element s of
// the step's four (s = 0, 1 -> fragment word 0, s = 2, 3 -> word 1). A and B use the same map. Q8: thread t takes
// weights 8t .. 8t+7 (bytes 8t .. 8t+7); Q4: bytes 4t .. 4t+3, their low nibbles (weights 4t .. 4t+3) for step 0 and
// their high nibbles (weights 16+4t .. 16+4t+3) for step 1.
template <bool Q4>
__device__ __forceinline__ void k_slot(int k, int &t, int &j, int &s) {
    if (Q4) {
        j = k / 16, t = (k % 16) / 4, s = k % 4;
    } else {
        t = k / 8, j = (k % 8) / 4, s = k % 4;
    }
}

template <bool Q4, bool SF16>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ CUtensorMap wmap, GemvArgs a, int C) {
    constexpr int BB = Q4 ? 16 : 32;  // bytes of a 32-block
    constexpr int kChunk = chunk_blocks<Q4>();
    using ST = typename std::conditional<SF16, __half, float>::type;  // scales keep their input type in shared memory
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the rings must sit on a 1024-byte boundary of the shared window (the swizzle is a function of the address)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint8_t *ring = smem + kBarBytes;
    uint4 *frag = reinterpret_cast<uint4 *>(smem + kBarBytes + ring_bytes<Q4>());                        // [bps][3][4m]
    ST *sc = reinterpret_cast<ST *>(smem + kBarBytes + ring_bytes<Q4>() + frag_bytes(a.bps, a.m));      // [kRows][bps+1]
    const int fl = 4 * a.m;  // fragment lanes stored per block and part
    float *red = reinterpret_cast<float *>(ring);  // reuses the rings once every warp has finished its main loop
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int crank = int(blockIdx.x) % C;
    const int64_t row0 = int64_t(blockIdx.x / C) * kRows;
    const int b0 = crank * a.bps;
    const int nb = max(0, min(a.nblk, b0 + a.bps) - b0);  // this CTA's K slice: blocks b0 .. b0 + nb - 1
    const int nchunks = (nb + kChunk - 1) / kChunk;
    const int sstride = a.bps + 1;

    // this warp's ring and barriers: lane 0 copies the warp's 32 rows x 128 bytes of a chunk with one 2-D tensor copy
    // (rows past the end of the matrix arrive as zeros)
    uint64_t *wbar = bars + warp * kStages;
    uint8_t *wring = ring + size_t(warp) * kStages * kStageBytes;
    const int wrow0 = int(row0) + warp * kWarpRows;  // rows < 2^31 (launcher)
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) mbar_init(&wbar[s], 1);
        mbar_init_fence();
    }
    __syncwarp();
    pdl_enter();
    // chunk c of the slice into stage c % kStages (the box is always whole: a chunk past the slice's end reads the
    // next slice's bytes or the zero fill, which the compute loop does not use)
    auto issue = [&](int c) {
        if (lane == 0) {
            const int s = c % kStages;
            mbar_arrive_expect_tx(&wbar[s], kStageBytes);
            tensor_g2s_2d(wring + s * kStageBytes, &wmap, (b0 + c * kChunk) * BB, wrow0, &wbar[s]);
        }
    };
    for (int c = 0; c < kStages && c < nchunks; ++c) issue(c);

    // prologue 1: activation splits in B-fragment order, for the m activation rows. Pair (k, k+1) of row n in block
    // bi goes to lane 4n + t, word 2j + s/2, part p. Loads are issued in batches of 8 per thread before any of them
    // is used.
    constexpr int kBatch = 8;
    const int npairs = nb * 16 * a.m;
    for (int o0 = 0; o0 < npairs; o0 += kBatch * kThreads) {
        float2 v[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int o = o0 + i * kThreads + threadIdx.x;
            const int bi = o / (16 * a.m), rem = o % (16 * a.m), n = rem / 16, k = 2 * (rem % 16);
            v[i] = (o < npairs)
                       ? __ldg(reinterpret_cast<const float2 *>(a.x + int64_t(n) * a.cols + int64_t(b0 + bi) * 32 + k))
                       : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int o = o0 + i * kThreads + threadIdx.x;
            if (o < npairs) {
                const int bi = o / (16 * a.m), rem = o % (16 * a.m), n = rem / 16, k = 2 * (rem % 16);
                uint32_t hi, mid, lo;
                split3(v[i].x, v[i].y, hi, mid, lo);
                int tq, j, sq;
                k_slot<Q4>(k, tq, j, sq);
                const int ln = 4 * n + tq, wd = 2 * j + sq / 2;
                uint32_t *f = reinterpret_cast<uint32_t *>(frag + size_t(bi) * 3 * fl);
                f[(0 * fl + ln) * 4 + wd] = hi;
                f[(1 * fl + ln) * 4 + wd] = mid;
                f[(2 * fl + ln) * 4 + wd] = lo;
            }
        }
    }
    // prologue 2: the CTA's block scales [row][block], in batches of 8 loads per thread
    const int nsc = kRows * a.bps;
    const ST *sg = static_cast<const ST *>(a.scale);
    for (int o0 = 0; o0 < nsc; o0 += kBatch * kThreads) {
        ST v[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int o = o0 + i * kThreads + threadIdx.x;
            const int r = int(a.bdiv.div(uint32_t(o))), bi = o - r * a.bps;
            const int64_t gr = row0 + r;
            v[i] = (o < nsc && bi < nb && gr < a.rows) ? __ldg(sg + gr * a.nblk + b0 + bi) : ST(0.f);
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int o = o0 + i * kThreads + threadIdx.x;
            const int r = int(a.bdiv.div(uint32_t(o))), bi = o - r * a.bps;
            if (o < nsc) sc[r * sstride + bi] = v[i];
        }
    }
    __syncthreads();

    float acc[kTiles][4];
#pragma unroll
    for (int tt = 0; tt < kTiles; ++tt) acc[tt][0] = acc[tt][1] = acc[tt][2] = acc[tt][3] = 0.f;
    const ST *scw = sc + (warp * kWarpRows + g) * sstride;
    uint32_t parity = 0;  // bit s: phase parity of stage s
    bool ok = true;
    for (int c = 0; c < nchunks && ok; ++c) {
        const int s = c % kStages;
        if (!mbar_wait_warp(&wbar[s], (parity >> s) & 1u)) {
            ok = false;  // the partial sums of this warp are abandoned; the flag reports it
            break;
        }
        parity ^= 1u << s;
        const uint8_t *st = wring + s * kStageBytes;
        const int nbk = min(kChunk, nb - c * kChunk);
        for (int kb = 0; kb < nbk; ++kb) {
            const int b = c * kChunk + kb;
            const bool fv = lane < fl;  // lanes of rows >= m multiply zeros
            const uint4 z = make_uint4(0, 0, 0, 0);
            const uint4 x0 = fv ? frag[(size_t(b) * 3 + 0) * fl + lane] : z;
            const uint4 x1 = fv ? frag[(size_t(b) * 3 + 1) * fl + lane] : z;
            const uint4 x2 = fv ? frag[(size_t(b) * 3 + 2) * fl + lane] : z;
#pragma unroll
            for (int tt = 0; tt < kTiles; ++tt) {
                // A words [k16 step j][word]: rows g (ga) and g + 8 (gb) of the tile
                const int r = 16 * tt + g;
                uint32_t ga[2][2], gb[2][2];
                if constexpr (Q4) {
                    const uint32_t m4 = 0x0F0F0F0Fu;
                    const uint32_t wa = *reinterpret_cast<const uint32_t *>(st + swz(r, kb * BB + 4 * t));
                    const uint32_t wb = *reinterpret_cast<const uint32_t *>(st + swz(r + 8, kb * BB + 4 * t));
                    q4_to_bf16(wa & m4, ga[0][0], ga[0][1]);
                    q4_to_bf16((wa >> 4) & m4, ga[1][0], ga[1][1]);
                    q4_to_bf16(wb & m4, gb[0][0], gb[0][1]);
                    q4_to_bf16((wb >> 4) & m4, gb[1][0], gb[1][1]);
                } else {
                    const uint2 wa = *reinterpret_cast<const uint2 *>(st + swz(r, kb * BB + 8 * t));
                    const uint2 wb = *reinterpret_cast<const uint2 *>(st + swz(r + 8, kb * BB + 8 * t));
                    q8_to_bf16(wa.x, ga[0][0], ga[0][1]);
                    q8_to_bf16(wa.y, ga[1][0], ga[1][1]);
                    q8_to_bf16(wb.x, gb[0][0], gb[0][1]);
                    q8_to_bf16(wb.y, gb[1][0], gb[1][1]);
                }
                // two independent accumulation chains (k16 steps 0 and 1), smallest parts first
                float p0[4] = {0.f, 0.f, 0.f, 0.f}, p1[4] = {0.f, 0.f, 0.f, 0.f};
                mma_bf16(p0, ga[0][0], gb[0][0], ga[0][1], gb[0][1], x2.x, x2.y);
                mma_bf16(p1, ga[1][0], gb[1][0], ga[1][1], gb[1][1], x2.z, x2.w);
                mma_bf16(p0, ga[0][0], gb[0][0], ga[0][1], gb[0][1], x1.x, x1.y);
                mma_bf16(p1, ga[1][0], gb[1][0], ga[1][1], gb[1][1], x1.z, x1.w);
                mma_bf16(p0, ga[0][0], gb[0][0], ga[0][1], gb[0][1], x0.x, x0.y);
                mma_bf16(p1, ga[1][0], gb[1][0], ga[1][1], gb[1][1], x0.z, x0.w);
                const float sa = float(scw[(16 * tt) * sstride + b]), sb = float(scw[(16 * tt + 8) * sstride + b]);
                acc[tt][0] = fmaf(p0[0] + p1[0], sa, acc[tt][0]);
                acc[tt][1] = fmaf(p0[1] + p1[1], sa, acc[tt][1]);
                acc[tt][2] = fmaf(p0[2] + p1[2], sb, acc[tt][2]);
                acc[tt][3] = fmaf(p0[3] + p1[3], sb, acc[tt][3]);
            }
        }
        __syncwarp();
        if (c + kStages < nchunks) {
            if (lane == 0) fence_proxy_async();  // this stage's shared reads precede the copy that refills it
            issue(c + kStages);
        }
    }
    if (!ok) {
        // let the warp's other copies land (bounded) before the CTA's shared memory can be reused
        for (int s = 0; s < kStages; ++s) mbar_wait_warp(&wbar[s], (parity >> s) & 1u);
    }
    __syncthreads();  // every warp is done with its ring: it becomes the reduction buffer
    // D fragment: acc[tt][0..1] = rows 16 tt + g, tokens 2t, 2t+1; acc[tt][2..3] = row + 8
#pragma unroll
    for (int tt = 0; tt < kTiles; ++tt) {
        const int r = warp * kWarpRows + 16 * tt + g;
        red[(2 * t) * kRedPad + r] = acc[tt][0];
        red[(2 * t + 1) * kRedPad + r] = acc[tt][1];
        red[(2 * t) * kRedPad + r + 8] = acc[tt][2];
        red[(2 * t + 1) * kRedPad + r + 8] = acc[tt][3];
    }
    const bool clustered = C > 1;
    if (clustered) cg::this_cluster().sync();
    else __syncthreads();
    // rows [crank * kRows / C, (crank + 1) * kRows / C) of the group: the cluster's K slices added in rank order
    const int lo_r = crank * kRows / C, hi_r = (crank + 1) * kRows / C, span = hi_r - lo_r;
    for (int o = threadIdx.x; o < span * kTok; o += kThreads) {
        const int tok = o / span, r = lo_r + o % span;
        const int64_t grow = row0 + r;
        if (tok >= a.m || grow >= a.rows) continue;
        float v;
        if (clustered) {
            cg::cluster_group cl = cg::this_cluster();
            v = 0.f;
            for (int q = 0; q < C; ++q) v += cl.map_shared_rank(red, q)[tok * kRedPad + r];
        } else {
            v = red[tok * kRedPad + r];
        }
        float *yp = a.y + int64_t(tok) * a.ystride + grow;
        const float out = (a.bias ? __ldg(a.bias + grow) : 0.f) + v;
        *yp = a.accumulate ? *yp + out : out;
    }
    if (clustered) cg::this_cluster().sync();  // no CTA leaves while another still reads its shared memory
}

// ------------------------------------------------------------------ CUDA-core path for one or two activation rows
//
// Decode multiplies one (or, with classifier-free guidance, two) activation rows: then the tensor cores' N = 8 columns
// are mostly zeros and the cost is the code conversion. This path spends about 2.4 instructions per weight: lane l
// streams 16 consecutive code bytes of a row (512 contiguous bytes per warp instruction), converts them with the same
// exact bit-pattern trick, multiplies them by its activation values held in registers (reused for the 32 rows of a
// batch), and scales the block partial once. A CTA (8 warps) owns 32 rows; its warps (and the C CTAs of a cluster)
// split the rows' 512-byte chunks; each warp's 32 row partials are reduced across its lanes by a transpose butterfly
// (31 shuffles), then across the warps and the cluster in fixed order.
constexpr int kCcRows = 32;

// exact f32 value of each of the four int8 codes of `word`, minus nothing: q (via 2^23 + (q + 128) - (2^23 + 128))
__device__ __forceinline__ void q8_to_f32(uint32_t word, float2 &c01, float2 &c23) {
    const uint32_t u = word ^ 0x80808080u;
    const float2 m = make_float2(-8388736.0f, -8388736.0f);
    c01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)), __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541))), m);
    c23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)), __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543))), m);
}
// four 4-bit codes (one per byte, 0..15) -> their values code - 8, exact
__device__ __forceinline__ void q4_to_f32(uint32_t nib, float2 &c01, float2 &c23) {
    const float2 m = make_float2(-8388616.0f, -8388616.0f);  // 2^23 + 8
    c01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7540)), __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7541))), m);
    c23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7542)), __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7543))), m);
}

template <bool Q4, bool SF16, int M>
__global__ void __launch_bounds__(kThreads, 2) gemv_cc_kernel(GemvArgs a, int C) {
    constexpr int NX = Q4 ? 32 : 16;  // activation values per lane per chunk
    constexpr int RB = 4;             // rows per batch (reduced across the warp together)
    __shared__ float red[kWarps][M][kCcRows];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int crank = int(blockIdx.x) % C;
    const int64_t row0 = int64_t(blockIdx.x / C) * kCcRows;
    const int64_t rowbytes = Q4 ? a.cols / 2 : a.cols;
    const int nchunk = int((rowbytes + 511) / 512);
    const int64_t last = a.rows - 1 - row0;  // rows r > last read row `last` (their sums are dropped)
    pdl_enter();
    // rows (b * RB + (lane % RB)) of batch b, per activation row: this lane's share of the warp's partial sums
    float tot[kCcRows / RB][M];
#pragma unroll
    for (int b = 0; b < kCcRows / RB; ++b)
#pragma unroll
        for (int t = 0; t < M; ++t) tot[b][t] = 0.f;
    for (int ci = crank * kWarps + warp; ci < nchunk; ci += kWarps * C) {
        const int64_t cb = int64_t(ci) * 512 + lane * 16;  // this lane's 16 bytes of every row
        const bool valid = cb < rowbytes;                 // a row's last chunk may be partial (rowbytes % 16 == 0)
        const int64_t blk = Q4 ? cb / 16 : cb / 32;       // the 32-block of these bytes
        const int64_t k0 = Q4 ? blk * 32 : cb;            // first activation index they multiply
        float2 xv[M][NX / 2];
#pragma unroll
        for (int t = 0; t < M; ++t)
#pragma unroll
            for (int q = 0; q < NX / 4; ++q) {
                const float4 v = valid ? __ldg(reinterpret_cast<const float4 *>(a.x + int64_t(t) * a.cols + k0) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                xv[t][2 * q] = make_float2(v.x, v.y);
                xv[t][2 * q + 1] = make_float2(v.z, v.w);
            }
        // the batch's 8 rows of codes and scales, double-buffered: batch b + 1 is requested before batch b is used
        // one 64-bit base per batch, 32-bit row offsets (rows of a CTA span < 2^31 bytes: launcher)
        const uint8_t *wcol = a.w + row0 * rowbytes + cb;
        const uint8_t *scol = static_cast<const uint8_t *>(a.scale) + (row0 * a.nblk + blk) * (SF16 ? 2 : 4);
        const uint32_t wstep = uint32_t(rowbytes), sstep = uint32_t(a.nblk * (SF16 ? 2 : 4));
        auto fetch = [&](int b, uint4 (&w)[RB], float (&sc)[RB]) {
#pragma unroll
            for (int r = 0; r < RB; ++r) {
                const uint32_t rr = uint32_t(b * RB + r <= last ? b * RB + r : last);
                w[r] = valid ? __ldcs(reinterpret_cast<const uint4 *>(wcol + rr * wstep)) : make_uint4(0, 0, 0, 0);
                sc[r] = valid ? load_scale<SF16>(scol + rr * sstep, 0) : 0.f;
            }
        };
        // the batch's 8 row partials of this warp, per activation row: lane l ends with row l % RB (all lanes of a
        // row agree)
        auto batch = [&](const uint4 (&wb)[RB], const float (&sb)[RB], float (&out)[M]) {
            float acc[RB][M];
#pragma unroll
            for (int r = 0; r < RB; ++r) {
                const uint32_t wd[4] = {wb[r].x, wb[r].y, wb[r].z, wb[r].w};
                float2 p[M][2];
#pragma unroll
                for (int t = 0; t < M; ++t) p[t][0] = p[t][1] = make_float2(0.f, 0.f);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float2 c01, c23;
                    if (Q4) {
                        // word i: codes 4i..4i+3 (low nibbles) and 16+4i..16+4i+3 (high nibbles)
                        float2 h01, h23;
                        q4_to_f32(wd[i] & 0x0F0F0F0Fu, c01, c23);
                        q4_to_f32((wd[i] >> 4) & 0x0F0F0F0Fu, h01, h23);
#pragma unroll
                        for (int t = 0; t < M; ++t) {
                            p[t][0] = __ffma2_rn(c01, xv[t][2 * i], p[t][0]);
                            p[t][1] = __ffma2_rn(c23, xv[t][2 * i + 1], p[t][1]);
                            p[t][0] = __ffma2_rn(h01, xv[t][8 + 2 * i], p[t][0]);
                            p[t][1] = __ffma2_rn(h23, xv[t][8 + 2 * i + 1], p[t][1]);
                        }
                    } else {
                        q8_to_f32(wd[i], c01, c23);
#pragma unroll
                        for (int t = 0; t < M; ++t) {
                            p[t][0] = __ffma2_rn(c01, xv[t][2 * i], p[t][0]);
                            p[t][1] = __ffma2_rn(c23, xv[t][2 * i + 1], p[t][1]);
                        }
                    }
                }
#pragma unroll
                for (int t = 0; t < M; ++t) {
                    const float2 q = __fadd2_rn(p[t][0], p[t][1]);
                    acc[r][t] = (q.x + q.y) * sb[r];
                }
            }
            // transpose butterfly over lane bits 1..0 (lane l keeps row l % RB), then a plain sum over bits 2..4
#pragma unroll
            for (int t = 0; t < M; ++t) {
#pragma unroll
                for (int s = RB / 2; s >= 1; s >>= 1) {
                    const bool up = (lane & s) != 0;
#pragma unroll
                    for (int j = 0; j < s; ++j) {
                        const float send = up ? acc[j][t] : acc[j + s][t];
                        const float keep = up ? acc[j + s][t] : acc[j][t];
                        acc[j][t] = keep + __shfl_xor_sync(0xffffffffu, send, s);
                    }
                }
                float v = acc[0][t];
#pragma unroll
                for (int s = RB; s < 32; s <<= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
                out[t] = v;
            }
        };
        constexpr int NB = kCcRows / RB;  // batches per chunk (even)
        uint4 w0[RB], w1[RB];
        float s0[RB], s1[RB];
        fetch(0, w0, s0);
#pragma unroll 1
        for (int b = 0; b < NB; b += 2) {
            fetch(b + 1, w1, s1);
            float v[M];
            batch(w0, s0, v);
#pragma unroll
            for (int k = 0; k < NB; k += 2)
#pragma unroll
                for (int t = 0; t < M; ++t) tot[k][t] += b == k ? v[t] : 0.f;
            if (b + 2 < NB) fetch(b + 2, w0, s0);
            batch(w1, s1, v);
#pragma unroll
            for (int k = 1; k < NB; k += 2)
#pragma unroll
                for (int t = 0; t < M; ++t) tot[k][t] += b + 1 == k ? v[t] : 0.f;
        }
    }
    if (lane < RB) {
#pragma unroll
        for (int b = 0; b < kCcRows / RB; ++b)
#pragma unroll
            for (int t = 0; t < M; ++t) red[warp][t][b * RB + lane] = tot[b][t];
    }
    __syncthreads();
    // the CTA's rows: sum of the warps in order; then the cluster's CTAs in rank order
    float *cta = &red[0][0][0];
    if (threadIdx.x < M * kCcRows) {
        const int t = threadIdx.x / kCcRows, r = threadIdx.x % kCcRows;
        float v = red[0][t][r];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) v += red[w][t][r];
        __syncwarp();
        cta[t * kCcRows + r] = v;  // red[0] is read above by this thread only
    }
    const bool clustered = C > 1;
    if (clustered) cg::this_cluster().sync();
    else __syncthreads();
    const int lo_r = crank * kCcRows / C, hi_r = (crank + 1) * kCcRows / C, span = hi_r - lo_r;
    if (threadIdx.x < M * span) {
        const int t = threadIdx.x / span, r = lo_r + threadIdx.x % span;
        const int64_t grow = row0 + r;
        if (t < a.m && grow < a.rows) {
            float v;
            if (clustered) {
                cg::cluster_group cl = cg::this_cluster();
                v = 0.f;
                for (int q = 0; q < C; ++q) v += cl.map_shared_rank(cta, q)[t * kCcRows + r];
            } else {
                v = cta[t * kCcRows + r];
            }
            float *yp = a.y + int64_t(t) * a.ystride + grow;
            const float out = (a.bias ? __ldg(a.bias + grow) : 0.f) + v;
            *yp = a.accumulate ? *yp + out : out;
        }
    }
    if (clustered) cg::this_cluster().sync();
}

// The same arithmetic with the rows and the scales staged by tensor copies (no registers held for bytes in flight,
// no load latency inside the loop): a warp streams its 512-byte chunk of the CTA's 16 rows as two copies of 8 rows
// (up to three in flight over the warp's chunks) and the chunk's block scales of the 16 rows as one copy issued with
// the chunk's first rows.
constexpr int kRowBatch = 8;              // rows per tensor copy
constexpr int kRowsCta = 16;              // rows per CTA: [12288, 4096] makes 768 CTAs, 2.6 waves of 2 per SM
constexpr int kRowStages = 2;             // copies in flight per warp (a warp of [rows, 4096] Q8 or Q4 has two)
constexpr int kRowBox = kRowBatch * 512;  // 4 KB
constexpr int kRowCopies = kRowsCta / kRowBatch;  // copies per chunk
// Blocks of a 512-byte row chunk: 16 (Q8, 32 bytes a block) or 32 (Q4, 16 bytes a block); their scales for the CTA's rows.
template <bool Q4> __host__ __device__ constexpr int chunk_scales() { return Q4 ? 32 : 16; }
// shared-memory reads by address (ld.shared): the staging rings sit behind a realigned pointer
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
template <typename ST> __device__ __forceinline__ float lds_scale(uint32_t a);
template <> __device__ __forceinline__ float lds_scale<__half>(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return __half2float(__ushort_as_half(v));
}
template <> __device__ __forceinline__ float lds_scale<float>(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
template <bool Q4, bool SF16> __host__ __device__ constexpr int scale_box() { return kRowsCta * chunk_scales<Q4>() * (SF16 ? 2 : 4); }
template <bool Q4, bool SF16, int M> __host__ __device__ constexpr size_t rows_smem() {  // + row partials of two groups
    return 256 + size_t(kWarps) * (kRowStages * kRowBox + 2 * scale_box<Q4, SF16>()) + size_t(2) * kWarps * M * kRowsCta * 4 + 128;
}

// Q8: lane l holds bytes 16 l .. 16 l + 15 of every row of the chunk (codes of half a block); Q4: the same 16 bytes
// are one whole block (byte j: element j in the low nibble, element j + 16 in the high nibble), so the lane keeps 32
// activation values and one scale per row.
//
// Row groups of kRowsCta rows: a cluster of C CTAs splits one group's chunks (C > 1, one group per cluster), or a
// persistent CTA (C = 1) takes groups blockIdx.x, + gridDim.x, ... and each warp's copy stream runs on across its
// groups, so the copies of the next group are in flight while the current one is reduced and written.
template <bool Q4, bool SF16, int M>
__global__ void __launch_bounds__(kThreads, (!Q4 && M == 1) ? 3 : M <= 2 ? 2 : 1) gemv_rows_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                 const __grid_constant__ CUtensorMap smap, GemvArgs a, int C) {
    using ST = typename std::conditional<SF16, __half, float>::type;
    constexpr int SB = scale_box<Q4, SF16>();
    constexpr int BPC = chunk_scales<Q4>();  // scales per row of a chunk
    constexpr int EPL = Q4 ? 32 : 16;        // weights (and activation values) per lane per row
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *wbar = reinterpret_cast<uint64_t *>(smem) + warp * kRowStages;
    uint8_t *wring = smem + 256 + size_t(warp) * (kRowStages * kRowBox + 2 * SB);
    uint8_t *sring = wring + kRowStages * kRowBox;  // two chunk instances' scales
    // row partials [2 (group parity)][kWarps][M][kRowsCta], after the rings
    float *redbuf = reinterpret_cast<float *>(smem + 256 + size_t(kWarps) * (kRowStages * kRowBox + 2 * SB));
    const int crank = int(blockIdx.x) % C;
    const int ngroups = int((a.rows + kRowsCta - 1) / kRowsCta);
    const int gstep = int(gridDim.x) / C;
    const int g0 = int(blockIdx.x) / C;
    const int ngm = g0 < ngroups ? (ngroups - g0 + gstep - 1) / gstep : 0;  // groups of this CTA
    const int64_t rowbytes = Q4 ? a.cols / 2 : a.cols;
    const int nchunk = int((rowbytes + 511) / 512);
    const int c0 = crank * kWarps + warp, cstep = kWarps * C;
    const int nmine = c0 < nchunk ? (nchunk - c0 + cstep - 1) / cstep : 0;  // chunks of this warp in every group
    const int upg = nmine * kRowCopies;                                       // units (copies of 8 rows) per group
    const int units = ngm * upg;
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kRowStages; ++s) mbar_init(&wbar[s], 1);
        mbar_init_fence();
    }
    __syncwarp();
    pdl_enter();
    // unit u: group g0 + (u / upg) gstep, chunk instance ck = u / kRowCopies (chunk c0 + (ck % nmine) cstep), rows
    // 8 (u % kRowCopies) .. + 7 of the group, into stage u % kRowStages; the first unit of a chunk instance also brings
    // the chunk's scales of the group's rows into scale buffer ck % 2
    auto issue = [&](int u) {
        if (lane == 0) {
            const int s = u % kRowStages, ck = u / kRowCopies, ci = c0 + (ck % nmine) * cstep;
            const int row0 = (g0 + (u / upg) * gstep) * kRowsCta;
            const bool with_scales = u % kRowCopies == 0;
            mbar_arrive_expect_tx(&wbar[s], kRowBox + (with_scales ? SB : 0));
            tensor_g2s_2d(wring + s * kRowBox, &wmap, ci * 128, row0 + (u % kRowCopies) * kRowBatch, &wbar[s]);
            if (with_scales) tensor_g2s_2d(sring + (ck & 1) * SB, &smap, ci * BPC, row0, &wbar[s]);
        }
    };
    for (int u = 0; u < kRowStages && u < units; ++u) issue(u);
    uint32_t parity = 0;
    bool ok = true;
    const bool clustered = C > 1;
    float2 xv[M][EPL / 2];  // this lane's activation values of its chunk (kept across groups when the warp has one chunk)
    for (int gi = 0; gi < ngm; ++gi) {
        const int row0 = (g0 + gi * gstep) * kRowsCta;
        float tot[kRowCopies][M];
#pragma unroll
        for (int b = 0; b < kRowCopies; ++b)
#pragma unroll
            for (int t = 0; t < M; ++t) tot[b][t] = 0.f;
        for (int k = 0; k < nmine && ok; ++k) {
            const int ck = gi * nmine + k;
            const int64_t cb = int64_t(c0 + k * cstep) * 512 + lane * 16;  // this lane's 16 bytes of every row
            const bool valid = cb < rowbytes;
            const int64_t e0 = Q4 ? 2 * cb : cb;  // its first weight's column
            if (gi == 0 || nmine > 1) {
#pragma unroll
                for (int t = 0; t < M; ++t)
#pragma unroll
                    for (int q = 0; q < EPL / 4; ++q) {
                        const float4 v = valid && t < a.m ? __ldg(reinterpret_cast<const float4 *>(a.x + int64_t(t) * a.cols + e0) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                        xv[t][2 * q] = make_float2(v.x, v.y);
                        xv[t][2 * q + 1] = make_float2(v.z, v.w);
                    }
            }
            const uint32_t scs = smem_addr(reinterpret_cast<const ST *>(sring + (ck & 1) * SB) + (Q4 ? lane : lane >> 1));  // [kRowsCta rows][BPC blocks]
#pragma unroll 1
            for (int b = 0; b < kRowCopies; ++b) {
                const int u = ck * kRowCopies + b, s = u % kRowStages;
                if (!mbar_wait_warp(&wbar[s], (parity >> s) & 1u)) {
                    ok = false;
                    break;
                }
                parity ^= 1u << s;
                const uint32_t st = smem_addr(wring + s * kRowBox + lane * 16);
                float acc[kRowBatch][M];
#pragma unroll
                for (int r = 0; r < kRowBatch; ++r) {
                    const uint4 w = lds_v4(st + r * 512);
                    const float sc = lds_scale<ST>(scs + uint32_t((b * kRowBatch + r) * BPC * sizeof(ST)));
                    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
                    float2 p[M][2];
#pragma unroll
                    for (int t = 0; t < M; ++t) p[t][0] = p[t][1] = make_float2(0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float2 c01, c23;
                        if constexpr (Q4) {
                            float2 h01, h23;
                            q4_to_f32(wd[i] & 0x0F0F0F0Fu, c01, c23);         // elements 4 i .. 4 i + 3
                            q4_to_f32((wd[i] >> 4) & 0x0F0F0F0Fu, h01, h23);  // elements 16 + 4 i .. 16 + 4 i + 3
#pragma unroll
                            for (int t = 0; t < M; ++t) {
                                p[t][0] = __ffma2_rn(c01, xv[t][2 * i], p[t][0]);
                                p[t][1] = __ffma2_rn(c23, xv[t][2 * i + 1], p[t][1]);
                                p[t][0] = __ffma2_rn(h01, xv[t][8 + 2 * i], p[t][0]);
                                p[t][1] = __ffma2_rn(h23, xv[t][8 + 2 * i + 1], p[t][1]);
                            }
                        } else {
                            q8_to_f32(wd[i], c01, c23);
#pragma unroll
                            for (int t = 0; t < M; ++t) {
                                p[t][0] = __ffma2_rn(c01, xv[t][2 * i], p[t][0]);
                                p[t][1] = __ffma2_rn(c23, xv[t][2 * i + 1], p[t][1]);
                            }
                        }
                    }
#pragma unroll
                    for (int t = 0; t < M; ++t) {
                        const float2 q = __fadd2_rn(p[t][0], p[t][1]);
                        acc[r][t] = (q.x + q.y) * sc;
                    }
                }
                __syncwarp();
                if (u + kRowStages < units) {
                    if (lane == 0) fence_proxy_async();  // this stage's (and the older scale buffer's) reads precede the refill
                    issue(u + kRowStages);
                }
                // transpose butterfly over lane bits 2..0 (lane l keeps row l % 8), then a plain sum over bits 3, 4
#pragma unroll
                for (int t = 0; t < M; ++t) {
#pragma unroll
                    for (int sh = kRowBatch / 2; sh >= 1; sh >>= 1) {
                        const bool up = (lane & sh) != 0;
#pragma unroll
                        for (int j = 0; j < sh; ++j) {
                            const float send = up ? acc[j][t] : acc[j + sh][t];
                            const float keep = up ? acc[j + sh][t] : acc[j][t];
                            acc[j][t] = keep + __shfl_xor_sync(0xffffffffu, send, sh);
                        }
                    }
                    float v = acc[0][t];
                    v += __shfl_xor_sync(0xffffffffu, v, 8);
                    v += __shfl_xor_sync(0xffffffffu, v, 16);
#pragma unroll
                    for (int bb = 0; bb < kRowCopies; ++bb) tot[bb][t] += b == bb ? v : 0.f;
                }
            }
        }
        // the group's row sums: warps' partials added in warp order, then (clusters) the CTAs' sums in rank order
        float *red = redbuf + (gi & 1) * (kWarps * M * kRowsCta);
        if (lane < kRowBatch) {
#pragma unroll
            for (int b = 0; b < kRowCopies; ++b)
#pragma unroll
                for (int t = 0; t < M; ++t) red[(warp * M + t) * kRowsCta + b * kRowBatch + lane] = tot[b][t];
        }
        __syncthreads();
        float *cta = red;  // warp 0's slots receive the CTA sums
        if (threadIdx.x < M * kRowsCta) {
            const int t = threadIdx.x / kRowsCta, r = threadIdx.x % kRowsCta;
            float v = red[t * kRowsCta + r];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) v += red[(w * M + t) * kRowsCta + r];
            cta[t * kRowsCta + r] = v;  // read above by this thread only
        }
        if (clustered) cg::this_cluster().sync();
        else __syncthreads();
        const int lo_r = crank * kRowsCta / C, hi_r = (crank + 1) * kRowsCta / C, span = hi_r - lo_r;
        if (threadIdx.x < M * span) {
            const int t = threadIdx.x / span, r = lo_r + threadIdx.x % span;
            const int64_t grow = row0 + r;
            if (t < a.m && grow < a.rows) {
                float v;
                if (clustered) {
                    cg::cluster_group cl = cg::this_cluster();
                    v = 0.f;
                    for (int q = 0; q < C; ++q) v += cl.map_shared_rank(cta, q)[t * kRowsCta + r];
                } else {
                    v = cta[t * kRowsCta + r];
                }
                float *yp = a.y + int64_t(t) * a.ystride + grow;
                const float out = (a.bias ? __ldg(a.bias + grow) : 0.f) + v;
                *yp = a.accumulate ? *yp + out : out;
            }
        }
        if (clustered) cg::this_cluster().sync();
    }
    if (!ok) {
        // let the warp's copies in flight land (bounded) before the CTA's shared memory can be released
        for (int s = 0; s < kRowStages; ++s) mbar_wait_warp(&wbar[s], (parity >> s) & 1u);
    }
}

struct GemvPlan {
    int C = 0;
    size_t smem = 0;
};

// The cluster size of a shape (rows, blocks per row) on the current device, chosen once and cached: one wave of
// resident CTAs, at least 4 blocks per slice, the shared memory within the device limit and the cluster co-resident.
template <bool Q4, bool SF16>
int plan_gemv(int64_t rows, int nblk, int m, GemvPlan &plan, const char *name) {
    static std::mutex mu;
    static std::map<std::tuple<int, int64_t, int, int>, GemvPlan> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch(name);
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(dev, rows, nblk, m);
    auto it = cache.find(key);
    if (it != cache.end()) {
        plan = it->second;
        return VOX_CUDA_OK;
    }
    auto kern = gemv_kernel<Q4, SF16>;
    // allow the device's whole opt-in shared memory and clusters above 8 (both per device, idempotent)
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin()) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return check_launch(name);
    const int64_t groups = (rows + kRows - 1) / kRows;
    // as many K slices as one wave of resident CTAs holds (at least 1, at most kMaxCluster)
    const int64_t want = resident_blocks((const void *)kern, kThreads, gemv_smem<Q4>((nblk + 7) / 8, SF16, m)) / groups;
    int C = int(want < 1 ? 1 : want < kMaxCluster ? want : kMaxCluster);
    while (C > 1 && (nblk + C - 1) / C < 4) --C;
    if (const char *e = std::getenv("VOX_CUDA_GEMV_SLICES")) {  // tuning: K slices per row group (1 .. 16)
        const int v = std::atoi(e);
        if (v >= 1 && v <= kMaxCluster) C = v;
    }
    // the fewest slices whose shared memory fits the device
    int c_min = 1;
    while (gemv_smem<Q4>((nblk + c_min - 1) / c_min, SF16, m) > size_t(smem_optin())) {
        if (++c_min > kMaxCluster) return set_error(VOX_CUDA_ERR_UNSUPPORTED, std::string(name) + ": matrix too wide");
    }
    if (C < c_min) C = c_min;
    for (;;) {
        const size_t smem = gemv_smem<Q4>((nblk + C - 1) / C, SF16, m);
        if (C == 1) {
            plan = GemvPlan{C, smem};
            break;
        }
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = unsigned(C);
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.gridDim = dim3(unsigned(groups * C));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters >= groups) {
            plan = GemvPlan{C, smem};
            break;
        }
        cudaGetLastError();
        if (C == c_min) {  // more row groups than co-resident clusters: take the fewest slices (several waves)
            if (clusters > 0 || C == 1) {
                plan = GemvPlan{C, smem};
                break;
            }
            return set_error(VOX_CUDA_ERR_UNSUPPORTED, std::string(name) + ": no co-resident cluster for this shape");
        }
        C = C - 1;  // not all clusters co-resident: fewer, longer slices
        if (C < c_min) C = c_min;
    }
    cache[key] = plan;
    return VOX_CUDA_OK;
}

// Cluster size of the CUDA-core path for a shape, cached: split the rows' 512-byte chunks over up to 8 CTAs so that
// one wave of resident CTAs is filled, every warp keeping at least one chunk, all clusters co-resident.
template <bool Q4, bool SF16, int M>
int plan_cc(int64_t rows, int64_t rowbytes, int &C_out, const char *name) {
    static std::mutex mu;
    static std::map<std::tuple<int, int64_t, int64_t>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch(name);
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(dev, rows, rowbytes);
    auto it = cache.find(key);
    if (it != cache.end()) {
        C_out = it->second;
        return VOX_CUDA_OK;
    }
    auto kern = gemv_cc_kernel<Q4, SF16, M>;
    const int64_t groups = (rows + kCcRows - 1) / kCcRows;
    const int64_t nchunk = (rowbytes + 511) / 512;
    const int64_t slots = resident_blocks((const void *)kern, kThreads, 0);
    int64_t c = slots / groups;
    if (c > nchunk / kWarps) c = nchunk / kWarps;
    if (c > 8) c = 8;
    int C = int(c < 1 ? 1 : c);
    while (C > 1) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = unsigned(C);
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.gridDim = dim3(unsigned(groups * C));
        cfg.blockDim = dim3(kThreads);
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters > 0) break;
        cudaGetLastError();
        --C;
    }
    cache[key] = C;
    C_out = C;
    return VOX_CUDA_OK;
}

template <bool Q4, bool SF16, int M>
int launch_cc(const GemvArgs &a, cudaStream_t st, const char *name) {
    int C = 1;
    const int rc = plan_cc<Q4, SF16, M>(a.rows, Q4 ? a.cols / 2 : a.cols, C, name);
    if (rc != VOX_CUDA_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(unsigned((a.rows + kCcRows - 1) / kCcRows * C));
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    int na = 0;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = unsigned(C);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    if (cudaLaunchKernelEx(&cfg, gemv_cc_kernel<Q4, SF16, M>, a, C) != cudaSuccess) return check_launch(name);
    return VOX_CUDA_OK;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// The 2-D tensor maps of a weight matrix, cached per device, address, shape and layout (zero fill past the edges):
//   kMmaBoxes: uint8 elements [rows][rowbytes], box 16 rows x 128 bytes, 128-byte swizzle (the MMA path's fragments);
//   kRowBoxes: 4-byte elements [rows][rowbytes / 4], box 8 rows x 512 bytes (the CUDA-core path reads rows in order);
//   kScaleBoxes / kScaleBoxes32: the block scales [rows][nblk] (2- or 4-byte elements, esize), box kRowsCta rows x 16
//   (Q8) or 32 (Q4) blocks.
enum MapKind { kMmaBoxes = 0, kRowBoxes = 1, kScaleBoxes = 2, kScaleBoxes32 = 3 };
int weight_map(const void *base, int64_t rows, int64_t width, int kind, int esize, CUtensorMap &map, const char *name) {
    static std::mutex mu;
    static std::map<std::tuple<int, const void *, int64_t, int64_t, int, int>, CUtensorMap> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch(name);
    const auto key = std::make_tuple(dev, base, rows, width, kind, esize);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        map = it->second;
        return VOX_CUDA_OK;
    }
    auto fn = encode_fn();
    if (!fn) return set_error(VOX_CUDA_ERR_DEVICE, std::string(name) + ": cuTensorMapEncodeTiled is not available");
    // width: bytes per row (kMmaBoxes, kRowBoxes) or elements per row (kScaleBoxes)
    cuuint64_t dims[2], strides[1];
    cuuint32_t box[2];
    CUtensorMapDataType dt;
    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
    if (kind == kMmaBoxes) {
        dims[0] = cuuint64_t(width), strides[0] = cuuint64_t(width), box[0] = kChunkBytes, box[1] = kWarpRows;
        dt = CU_TENSOR_MAP_DATA_TYPE_UINT8, sw = CU_TENSOR_MAP_SWIZZLE_128B;
    } else if (kind == kRowBoxes) {
        dims[0] = cuuint64_t(width / 4), strides[0] = cuuint64_t(width), box[0] = 128, box[1] = 8;
        dt = CU_TENSOR_MAP_DATA_TYPE_UINT32;
    } else {  // scales: 16 (Q8) or 32 (Q4) blocks of 32 rows
        dims[0] = cuuint64_t(width), strides[0] = cuuint64_t(width * esize), box[0] = kind == kScaleBoxes32 ? 32 : 16, box[1] = kRowsCta;
        dt = esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    }
    dims[1] = cuuint64_t(rows);
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(&map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VOX_CUDA_ERR_ARG, std::string(name) + ": weight tensor map rejected (code " + std::to_string(int(r)) + ")");
    if (cache.size() > 4096) cache.clear();  // bounded: weights are long-lived, so the map rarely refills
    cache[key] = map;
    return VOX_CUDA_OK;
}

// Tensor-copy staging of the CUDA-core path (VOX_CUDA_GEMV_TMA=0 keeps the register-staged kernel, for comparisons).
bool tma_rows_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("VOX_CUDA_GEMV_TMA");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <bool Q4, bool SF16, int M>
int launch_rows(const GemvArgs &a, cudaStream_t st, const char *name) {
    auto kern = gemv_rows_kernel<Q4, SF16, M>;
    constexpr size_t smem_bytes = rows_smem<Q4, SF16, M>();
    const int64_t rowbytes = Q4 ? a.cols / 2 : a.cols;
    static std::mutex mu;
    static std::map<std::tuple<int, int64_t, int64_t>, std::pair<int, int64_t>> plans;  // (C, grid)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch(name);
    int C = 1;
    int64_t grid = 1;
    {
        std::lock_guard<std::mutex> lk(mu);
        const auto key = std::make_tuple(dev, a.rows, a.cols);
        auto it = plans.find(key);
        if (it != plans.end()) {
            C = it->second.first;
            grid = it->second.second;
        } else {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_bytes)) != cudaSuccess)
                return check_launch(name);
            const int64_t groups = (a.rows + kRowsCta - 1) / kRowsCta, nchunk = (rowbytes + 511) / 512;
            const int64_t slots = resident_blocks((const void *)kern, kThreads, smem_bytes);
            int64_t c = slots / groups;
            if (c > nchunk / kWarps) c = nchunk / kWarps;
            C = int(c < 1 ? 1 : c > 8 ? 8 : c);
            while (C > 1) {  // all clusters co-resident
                cudaLaunchConfig_t q = {};
                cudaLaunchAttribute at;
                at.id = cudaLaunchAttributeClusterDimension;
                at.val.clusterDim.x = unsigned(C), at.val.clusterDim.y = 1, at.val.clusterDim.z = 1;
                q.gridDim = dim3(unsigned(groups * C)), q.blockDim = dim3(kThreads), q.dynamicSmemBytes = smem_bytes;
                q.attrs = &at, q.numAttrs = 1;
                int clusters = 0;
                if (cudaOccupancyMaxActiveClusters(&clusters, kern, &q) == cudaSuccess && clusters > 0) break;
                cudaGetLastError();
                --C;
            }
            // one group per cluster (C > 1), or persistent CTAs, one resident wave, over the groups (C = 1)
            grid = C > 1 ? groups * C : (groups < slots ? groups : (slots > 0 ? slots : 1));
            plans[key] = std::make_pair(C, grid);
        }
    }
    CUtensorMap wmap, smap;
    int rc = weight_map(a.w, a.rows, rowbytes, kRowBoxes, 1, wmap, name);
    if (rc == VOX_CUDA_OK) rc = weight_map(a.scale, a.rows, a.nblk, Q4 ? kScaleBoxes32 : kScaleBoxes, SF16 ? 2 : 4, smap, name);
    if (rc != VOX_CUDA_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = st;
    int na = 0;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = unsigned(C);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    if (cudaLaunchKernelEx(&cfg, kern, wmap, smap, a, C) != cudaSuccess) return check_launch(name);
    return VOX_CUDA_OK;
}

template <bool Q4, bool SF16>
int launch_gemv(const GemvArgs &base, int64_t m_total, cudaStream_t st, const char *name) {
    if ((base.rows + kRows - 1) / kRows * kMaxCluster > int64_t(0x7FFFFFFF) || base.rows + kRows > int64_t(0x7FFFFFFF))
        return set_error(VOX_CUDA_ERR_ARG, std::string(name) + ": too many rows");
    CUtensorMap wmap;
    int rc = weight_map(base.w, base.rows, Q4 ? base.cols / 2 : base.cols, kMmaBoxes, 1, wmap, name);
    if (rc != VOX_CUDA_OK) return rc;
    auto kern = gemv_kernel<Q4, SF16>;
    for (int64_t i0 = 0; i0 < m_total; i0 += kTok) {  // activation rows in launches of 8
        GemvArgs a = base;
        a.m = int(m_total - i0 < kTok ? m_total - i0 : kTok);
        a.x = base.x + i0 * base.cols;
        a.y = base.y + i0 * base.ystride;
        if (a.m <= 2) {  // one or two activation rows: the CUDA-core path with tensor-copy staging (measured faster)
            const bool staged = (a.nblk * (SF16 ? 2 : 4)) % 16 == 0 && aligned16(a.scale) && tma_rows_enabled();
            if (staged) {
                rc = a.m == 1 ? launch_rows<Q4, SF16, 1>(a, st, name) : launch_rows<Q4, SF16, 2>(a, st, name);
                if (rc != VOX_CUDA_OK) return rc;
                continue;
            }
            if constexpr (!Q4) {  // register-staged Q8 where the scale rows are not 16-byte strided
                rc = a.m == 1 ? launch_cc<Q4, SF16, 1>(a, st, name) : launch_cc<Q4, SF16, 2>(a, st, name);
                if (rc != VOX_CUDA_OK) return rc;
                continue;
            }
        }
        if (a.m <= 4) {  // three or four activation rows: the same kernel with four (measured 1.5-1.7 x the MMA kernel)
            const bool staged = (a.nblk * (SF16 ? 2 : 4)) % 16 == 0 && aligned16(a.scale) && tma_rows_enabled();
            if (staged) {
                rc = launch_rows<Q4, SF16, 4>(a, st, name);
                if (rc != VOX_CUDA_OK) return rc;
                continue;
            }
        }
        GemvPlan plan;
        rc = plan_gemv<Q4, SF16>(base.rows, base.nblk, a.m, plan, name);
        if (rc != VOX_CUDA_OK) return rc;
        const int C = plan.C;
        a.bps = (a.nblk + C - 1) / C;
        a.bdiv = FastDiv(uint32_t(a.bps));
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[2];
        cfg.gridDim = dim3(unsigned((base.rows + kRows - 1) / kRows * C));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = plan.smem;
        cfg.stream = st;
        int na = 0;
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = unsigned(C);
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
        if (pdl_enabled()) {
            attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[na].val.programmaticStreamSerializationAllowed = 1;
            ++na;
        }
        cfg.attrs = attr;
        cfg.numAttrs = na;
        if (cudaLaunchKernelEx(&cfg, kern, wmap, a, C) != cudaSuccess) return check_launch(name);
    }
    return check_launch(name);
}

int gemv_entry(bool q4, const void *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y,
               int64_t rows, int64_t cols, int64_t m, int accumulate, void *stream, const char *name) {
    VOX_REQUIRE(scale_dtype == VOX_CUDA_F32 || scale_dtype == VOX_CUDA_F16, std::string(name) + ": scale dtype must be F32 or F16");
    VOX_REQUIRE(rows >= 0 && cols > 0 && m >= 0 && cols % 32 == 0, std::string(name) + ": bad shape (cols must be a multiple of 32)");
    if (rows == 0 || m == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(w && scale && x && y, std::string(name) + ": NULL pointer");
    VOX_REQUIRE(aligned16(w) && aligned16(x), std::string(name) + ": w and x must be 16-byte aligned");
    VOX_REQUIRE(cols / 32 < (int64_t(1) << 31), std::string(name) + ": too many columns");
    GemvArgs a{};
    a.w = static_cast<const uint8_t *>(w);
    a.scale = scale;
    a.bias = bias;
    a.x = x;
    a.y = y;
    a.rows = rows;
    a.cols = cols;
    a.ystride = rows;
    a.accumulate = accumulate != 0;
    a.nblk = int(cols / 32);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool f16 = scale_dtype == VOX_CUDA_F16;
    if (q4) return f16 ? launch_gemv<true, true>(a, m, st, name) : launch_gemv<true, false>(a, m, st, name);
    return f16 ? launch_gemv<false, true>(a, m, st, name) : launch_gemv<false, false>(a, m, st, name);
}

}  // namespace

int gemv_take_device_error(unsigned int *flags) { return take_device_error(flags); }

}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_gemv_q8(const int8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y, int64_t rows,
                     int64_t cols, int64_t m, int accumulate, void *stream) {
    return gemv_entry(false, w, scale, scale_dtype, bias, x, y, rows, cols, m, accumulate, stream, "vox_cuda_gemv_q8");
}

int vox_cuda_gemv_q4(const uint8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y, int64_t rows,
                     int64_t cols, int64_t m, int accumulate, void *stream) {
    return gemv_entry(true, w, scale, scale_dtype, bias, x, y, rows, cols, m, accumulate, stream, "vox_cuda_gemv_q4");
}

}  // extern "C"
