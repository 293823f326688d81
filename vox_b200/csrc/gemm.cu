// GEMM on the 5th-generation tensor cores: y[z][M][N] = x[z][M][K] . W[g][N][K]^T (+ bias) with a fused epilogue,
// bf16 operands, f32 accumulation in tensor memory. It replaces the projections Vox records as GEMM dispatches in its
// GPU F5 step (gpu_f5.cpp:287-322, gemm(): shaders/gemmb.comp:1-99, with its bias and GELU flags) and the grouped
// position convolutions' GEMMs (shaders/convgemm.comp).
//
// One CTA per SM (or a CTA pair on two SMs), persistent over output tiles of 128 rows x BN columns (BN 64, 128 or 256;
// pairs: 256 x 128 / 192 / 256), tiles with the same W columns taken by neighbouring CTAs so a weight tile is read from
// HBM once and then from L2. Six warps:
//   warp 0      tensor copies (TMA): for every K step of 64, the x tile [128][64] and the W tile [BN][64], both in the
//               128-byte swizzle, into a ring of STAGES shared-memory stages (mbarrier full/empty pairs);
//   warp 1      issues tcgen05.mma (M 128, N BN, K 16; four per K step) through one elected lane into one of two TMEM
//               accumulators and commits each stage back to the copy warp, and each finished tile to the epilogue;
//   warps 2..5  the epilogue: each thread reads its output row from TMEM (warp w reads lanes 32 (w % 4) ..), applies
//               bias / RoPE / GELU, stages the block in shared memory and writes it with a tensor store; the
//               accumulator goes back to the MMA warp, which meanwhile has started the next tile in the other
//               accumulator.
// Copies and MMAs are issued by the whole converged warp with one elected lane (measured: 347 -> 149 clocks to issue
// a K step's four MMAs and commit, against a single-lane branch). Eight epilogue warps (two a lane quadrant, alternate
// 32-column chunks) measured no faster in the F5 step and slower on long K (fewer copy stages fit). Every wait is
// bounded; a wait that gives up sets the device error flag and the CTA winds down (its copies and MMAs in flight are
// waited for, bounded, before its shared and tensor memory are released). No copy is broadcast across a cluster.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "gemm.cuh"
#include "sfu.cuh"
#include "tc.cuh"

namespace voxcuda {
namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kGemmThreads = 192;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB

template <int BN> struct Cfg {
    static constexpr int STAGES = BN == 256 ? 4 : BN == 128 ? 5 : 7;
    static constexpr uint32_t SWB = BN == 256 ? 4096 : 8192;  // epilogue staging bytes a warp
    static constexpr uint32_t B_BYTES = BN * kBK * 2;
    static constexpr uint32_t STAGE = kABytes + B_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
    static constexpr size_t SMEM = size_t(STAGES) * STAGE + 1024 + 256 + 4 * SWB + 4 * 1024;  // + epilogue staging and bias
};


// Output tile t: row block t % mt (the fastest, so neighbouring CTAs share a W tile), column block ni, plane z.
struct Tile {
    int m0, ni, z, zb, zg;
};
__device__ __forceinline__ Tile tile_of(int t, int mt, int nt, int groups) {
    Tile r;
    const int mi = t % mt, rest = t / mt;
    r.m0 = mi * kBM;
    r.ni = rest % nt;
    r.z = rest / nt;
    r.zb = r.z / groups;
    r.zg = r.z - r.zb * groups;
    return r;
}

constexpr uint32_t kStageWarpBytes = 32 * 128;  // one epilogue staging block: a warp's 32 rows x 32 columns (f32), 4 KB

// The epilogue of 32 consecutive columns [c0, c0 + 32) of the warp's 32 output rows m32 .. m32 + 31 (thread lane holds
// row m32 + lane; acc: f32 bit patterns): bias / RoPE / GELU on the registers, then the block passes through the warp's
// staging area in shared memory (16-byte chunk c of row r at chunk c ^ (r % 8): conflict-free both ways) so that each
// store instruction writes whole 128-byte row segments of y instead of 32 scattered pieces.
// Per-tile inputs of the epilogue, loaded before the accumulator is waited for (so the chunk loop makes no global
// loads): the tile's bias columns in the warp's shared-memory slot, and (RoPE) the thread's row of the cos / sin table
// in registers.
struct EpiPre {
    const float *bias_s;  // this warp's copy of bias[n0 .. n0 + BN) (shared memory), or nullptr
    float2 cs[32];        // RoPE: cs[row % frames][0 .. hd / 2) (hd = 64)
};

template <int EPI>
__device__ __forceinline__ void epi_prepare(const GemmArgs &g, int n0, int bn, int zg, int row, int lane, float *bias_s, EpiPre &pre) {
    pre.bias_s = nullptr;
    if (g.bias) {
        __syncwarp();  // the previous tile's readers are done with the slot
        for (int i = lane; i < bn; i += 32) bias_s[i] = n0 + i < g.N ? __ldg(g.bias + int64_t(zg) * g.N + n0 + i) : 0.f;
        __syncwarp();
        pre.bias_s = bias_s;
    }
    if constexpr (EPI == kEpiQkvRope) {
        const float2 *cs = g.cs + int64_t((row < g.M ? row : 0) % g.frames) * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) pre.cs[j] = __ldg(cs + j);
    }
}

// SWB: the warp's staging bytes; tensor stores rotate through SWB / block-size blocks (seq counts the warp's stores),
// so a block waits only for the store that used its buffer SWB / block-size stores before.
template <int EPI, uint32_t SWB>
__device__ __forceinline__ void epilogue32(const GemmArgs &g, const CUtensorMap *ty, const uint32_t (&acc)[32], int m32, int lane, int c0, int zb,
                                           int zg, uint32_t stg, uint32_t &seq, const EpiPre &pre, int cb) {
    const int row = m32 + lane;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(acc[i]);
    const int nv = min(32, g.N - c0);  // valid columns (warp-uniform)
    if (pre.bias_s) {  // tile columns cb .. cb + 31 (zeros past N)
        const float4 *b4 = reinterpret_cast<const float4 *>(pre.bias_s + cb);
#pragma unroll
        for (int q = 0; q < 8; ++q) {  // packed f32x2 adds (each rounded as the scalar add)
            const float4 bb = b4[q];
            const float2 lo = add2(make_float2(v[4 * q], v[4 * q + 1]), make_float2(bb.x, bb.y));
            const float2 hi = add2(make_float2(v[4 * q + 2], v[4 * q + 3]), make_float2(bb.z, bb.w));
            v[4 * q] = lo.x, v[4 * q + 1] = lo.y, v[4 * q + 2] = hi.x, v[4 * q + 3] = hi.y;
        }
    }
    if constexpr (EPI == kEpiQkvRope) {
        // q, k or v part, and the head (hd is 64 for this epilogue: gemm_plan checks it), without divisions
        const int part = c0 >= 2 * g.inner ? 2 : c0 >= g.inner ? 1 : 0, ci = c0 - part * g.inner, head = ci >> 6;
        if (part < 2 && head < g.rope_heads && row < g.M) {  // pairs (2j, 2j + 1) of the head, j = (ci % 64) / 2 ..
            const bool hi = (ci & 63) >= 32;                      // the head's second 32 columns: pairs 16 .. 31
            // (x0, x1) -> (x0 c - x1 s, x1 c + x0 s) (f5.cpp:696-701) as one packed multiply and one packed FMA a pair:
            // each output rounded once instead of three times; the bf16 output rounding is far larger than the difference
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float2 c = hi ? pre.cs[16 + j] : pre.cs[j];
                const float2 x = make_float2(v[2 * j], v[2 * j + 1]);
                const float2 r = fma2(x, make_float2(c.x, c.x), mul2(make_float2(x.y, x.x), make_float2(-c.y, c.y)));
                v[2 * j] = r.x, v[2 * j + 1] = r.y;
            }
        }
    } else if constexpr (EPI == kEpiGeluTanh || EPI == kEpiGeluTanhF32) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float2 r = gelu_tanh_f2(make_float2(v[2 * j], v[2 * j + 1]));
            v[2 * j] = r.x, v[2 * j + 1] = r.y;
        }
    } else if constexpr (EPI == kEpiGeluErf || EPI == kEpiGeluErfF32) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float2 r = gelu_erf_f2(make_float2(v[2 * j], v[2 * j + 1]));
            v[2 * j] = r.x, v[2 * j + 1] = r.y;
        }
    }
    constexpr bool F32OUT = EPI == kEpiF32 || EPI == kEpiGeluTanhF32 || EPI == kEpiGeluErfF32;
    constexpr int CH = F32OUT ? 8 : 4;             // 16-byte chunks a row
    constexpr int EPC = F32OUT ? 4 : 8;            // elements a chunk
    constexpr int RB = CH * 16;                    // staged row bytes
    const bool tst = g.tma_store != 0;
    constexpr uint32_t BOX = 32 * RB;              // staged block bytes
    constexpr int NB = int(SWB / BOX);             // staging buffers for tensor stores
    if (tst) {  // the store that last used this buffer has finished reading it (a no-op in lanes without stores)
        stg += (seq % uint32_t(NB)) * BOX;
        bulk_wait_read<NB - 1>();
        __syncwarp();
    }
    // registers -> staging (row = lane). For a tensor store the layout is the map's swizzle: 16-byte chunk c of row r at
    // c ^ (r % 8) (f32, 128-byte rows: the 128-byte swizzle) or c ^ ((r / 2) % 4) (bf16, 64-byte rows: the 64-byte
    // swizzle); both are free of bank conflicts for these writes.
    const int sw = F32OUT ? (lane & 7) : tst ? ((lane >> 1) & 3) : (lane & 3);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        uint4 w;
        if (F32OUT) w = make_uint4(__float_as_uint(v[4 * c]), __float_as_uint(v[4 * c + 1]), __float_as_uint(v[4 * c + 2]), __float_as_uint(v[4 * c + 3]));
        else w = make_uint4(pack_bf16(v[8 * c], v[8 * c + 1]), pack_bf16(v[8 * c + 2], v[8 * c + 3]), pack_bf16(v[8 * c + 4], v[8 * c + 5]),
                            pack_bf16(v[8 * c + 6], v[8 * c + 7]));
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(stg + lane * RB + ((c ^ sw) << 4)), "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w)
                     : "memory");
    }
    if (tst) {  // one tensor store (or add) of the 32 x 32 block; rows >= M and columns past the map's extent are clipped
        fence_proxy_async();
        __syncwarp();
        tma_store_3d_warp(ty, stg, int(int64_t(zg) * g.y_gstride) + c0, m32, zb, F32OUT && g.accumulate);
        ++seq;
        return;
    }
    __syncwarp();
    // staging -> y: each instruction covers 32 / CH rows, CH lanes a row (one 16-byte chunk each)
    constexpr int RPI = 32 / CH;
    const int c = lane % CH;
    const int64_t base = int64_t(zb) * g.y_bstride + int64_t(zg) * g.y_gstride + c0 + c * EPC;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int r = j * RPI + lane / CH;
        uint4 w;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                     : "r"(stg + r * RB + ((c ^ (r & (CH - 1))) << 4)) : "memory");
        const int gr = m32 + r;
        if (gr >= g.M) continue;
        const int64_t off = base + int64_t(gr) * g.ldy;
        const int nvc = min(EPC, nv - c * EPC);  // valid elements of this chunk
        if (nvc <= 0) continue;
        if (F32OUT) {
            float *y = reinterpret_cast<float *>(g.y) + off;
            float f[4] = {__uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w)};
            if (nvc == 4 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0) {
                if (g.accumulate) {
                    const float4 p = *reinterpret_cast<const float4 *>(y);
                    f[0] += p.x, f[1] += p.y, f[2] += p.z, f[3] += p.w;
                }
                *reinterpret_cast<float4 *>(y) = make_float4(f[0], f[1], f[2], f[3]);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (i < nvc) y[i] = g.accumulate ? y[i] + f[i] : f[i];
            }
        } else {
            uint16_t *y = reinterpret_cast<uint16_t *>(g.y) + off;
            if (nvc == 8 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0) {
                *reinterpret_cast<uint4 *>(y) = w;
            } else {
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (i < nvc) y[i] = uint16_t(ww[i / 2] >> (16 * (i & 1)));
            }
        }
    }
    __syncwarp();  // the staging area is reused by the next block
}

// One tiled copy issued by a whole converged warp through an elected lane, completing on `bar`; with expect_bytes > 0
// the lane first arrives on `bar` expecting that many bytes (the whole stage).
__device__ __forceinline__ void tma_one_warp(uint64_t *bar, uint32_t expect_bytes, uint32_t dst, const CUtensorMap *map, int x, int y, int z) {
    asm volatile("{\n\t.reg .pred e, f;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.and.b32 f, %1, 0, e;\n\t"
                 "@f mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t"
                 "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%3, {%4, %5, %6}], [%0];\n\t}"
                 ::"r"(smem_addr(bar)), "r"(expect_bytes), "r"(dst), "l"(map), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// The epilogue of one accumulator: its 32-column chunks [0, nch) (thread = row m32 + lane; taddr: this warp's lanes,
// column 0), each loaded from tensor memory, finished and stored in turn. (Loading the next chunk while the current
// one is stored measured slower.)
template <int EPI, uint32_t SWB>
__device__ __forceinline__ void epilogue_tile(const GemmArgs &g, const CUtensorMap *ty, uint32_t taddr, int nch, int m32, int lane, int n0,
                                              int zb, int zg, uint32_t stg, uint32_t &seq, const EpiPre &pre) {
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + uint32_t(32 * c), r);
        tmem_wait_ld(r);
        epilogue32<EPI, SWB>(g, ty, r, m32, lane, n0 + 32 * c, zb, zg, stg, seq, pre, 32 * c);
    }
}

// F16: f16 x and W instead of bf16 (the quantized GEMM's two-pass form); same kernel, the MMA's operand type differs.
template <int BN, int EPI, bool F16 = false>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                                                                  const __grid_constant__ CUtensorMap ty, const GemmArgs g) {
    using C = Cfg<BN>;
    constexpr uint32_t kIdesc = F16 ? umma_idesc_f16(kBM, BN) : umma_idesc_bf16(kBM, BN);
    extern __shared__ uint8_t gemm_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t s0 = smem_addr(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE + 4 * C::SWB);
    uint64_t *empty = full + C::STAGES;
    uint64_t *tfull = empty + C::STAGES;  // [2]: accumulator a holds a finished tile
    uint64_t *tempty = tfull + 2;         // [2]: accumulator a has been read out
    uint64_t *drain = tempty + 2;         // wind-down: every MMA issued has completed
    uint32_t *tslot = reinterpret_cast<uint32_t *>(drain + 1);
    const uint32_t STG_BASE = s0 + C::STAGES * C::STAGE;  // the epilogue warps' staging areas (1024-byte aligned), then the barriers
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (g.M + kBM - 1) / kBM, nt = (g.N + BN - 1) / BN;
    const int tiles = mt * nt * g.batches * g.groups, kt = (g.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&tfull[0], 1);
        mbar_init(&tfull[1], 1);
        mbar_init(&tempty[0], 4);
        mbar_init(&tempty[1], 4);
        mbar_init(drain, 1);
        mbar_init_fence();
        tma_prefetch_desc(&ta);
        tma_prefetch_desc(&tb);
    }
    if (warp == 0) tmem_alloc(tslot, C::TMEM_COLS);  // (no kernel of this library co-resides with a GEMM CTA: shared memory)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // the previous grid is complete before the first read of its outputs and the first write of y (the copy warp waits
    // below, after its early weight copies)
    if (warp != 0 || !g.w_early) pdl_enter();
    const uint32_t tmem = *tslot;
    bool ok = true;

    if (warp == 0) {
        // ---- tensor copies. With w_early, the W tiles of the first tile's first STAGES K steps are requested before
        // the previous grid has ended (W is none of its outputs), so their latency overlaps that grid's tail.
        int pre = 0;
        if (g.w_early) {
            if (int(blockIdx.x) < tiles) {
                const Tile tl = tile_of(int(blockIdx.x), mt, nt, g.groups);
                pre = kt < C::STAGES ? kt : C::STAGES;
                for (int kc = 0; kc < pre; ++kc)
                    tma_one_warp(&full[kc], C::STAGE, s0 + uint32_t(kc) * C::STAGE + kABytes, &tb, kc * kBK, tl.ni * BN, tl.zg);
                __syncwarp();
            }
            pdl_enter();
        }
        uint32_t it = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            const Tile tl = tile_of(t, mt, nt, g.groups);
            for (int kc = 0; kc < kt; ++kc, ++it) {
                const int s = int(it % C::STAGES);
                const uint32_t u = it / C::STAGES;
                const uint32_t sa = s0 + uint32_t(s) * C::STAGE;
                if (int(it) < pre) {  // its W copy is in flight already (the stage's bytes expected): x only
                    tma_one_warp(&full[s], 0, sa, &ta, kc * kBK, tl.m0, tl.z);
                    __syncwarp();
                    continue;
                }
                if (!mbar_wait_warp(&empty[s], (u & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                tma_stage_warp(&full[s], C::STAGE, sa, &ta, kc * kBK, tl.m0, tl.z, sa + kABytes, &tb, kc * kBK, tl.ni * BN, tl.zg);
                __syncwarp();
            }
        }
        if (!ok) {  // wind-down: the copies this warp issued land before the CTA's shared memory is released
            const uint32_t last = it;  // stages [last - STAGES, last) may still be in flight
            for (uint32_t j = last > uint32_t(C::STAGES) ? last - C::STAGES : 0; j < last; ++j)
                mbar_wait_warp(&full[j % C::STAGES], (j / C::STAGES) & 1u);
        }
    } else if (warp == 1) {
        // ---- MMA issue
        uint32_t it = 0, tc = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
            const uint32_t a = tc & 1u, v = tc >> 1;
            if (!mbar_wait_warp(&tempty[a], (v & 1u) ^ 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t dcol = tmem + a * BN;
            for (int kc = 0; kc < kt; ++kc, ++it) {
                const int s = int(it % C::STAGES);
                const uint32_t u = it / C::STAGES;
                if (!mbar_wait_warp(&full[s], u & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                {  // the whole warp, one lane elected to issue (operands warp-uniform)
                    const uint32_t sa = s0 + uint32_t(s) * C::STAGE, sb = sa + kABytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        umma_bf16_warp(dcol, umma_desc(sa + 32 * k, 16, 1024), umma_desc(sb + 32 * k, 16, 1024), kIdesc, (kc | k) != 0);
                    umma_commit_warp(&empty[s]);  // the stage returns to the copy warp when these MMAs have read it
                }
                __syncwarp();
            }
            if (!ok) break;
            umma_commit_warp(&tfull[a]);
            __syncwarp();
        }
        if (!ok) {  // wind-down: every MMA issued completes before the tensor memory is released
            umma_commit_warp(drain);
            __syncwarp();
            mbar_wait_warp(drain, 0);
        }
    } else {
        // ---- epilogue: thread = output row 32 (warp % 4) + lane of the tile
        const int q = warp & 3;
        const uint32_t stg = STG_BASE + uint32_t(warp - 2) * C::SWB;
        float *bias_s = reinterpret_cast<float *>(smem + C::STAGES * C::STAGE + 4 * C::SWB + 256) + (warp - 2) * 256;
        uint32_t seq = 0;
        uint32_t tc = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
            const uint32_t a = tc & 1u, v = tc >> 1;
            const Tile tl = tile_of(t, mt, nt, g.groups);
            EpiPre pre;
            epi_prepare<EPI>(g, tl.ni * BN, BN, tl.zg, tl.m0 + 32 * q + lane, lane, bias_s, pre);
            if (!mbar_wait_warp(&tfull[a], v & 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int n0 = tl.ni * BN, nch = min(BN, g.N - n0 + 31) / 32;  // chunks holding columns < N
            epilogue_tile<EPI, C::SWB>(g, &ty, tmem + (uint32_t(32 * q) << 16) + a * BN, nch, tl.m0 + 32 * q, lane, n0, tl.zb, tl.zg, stg, seq, pre);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);
        }
        if (g.tma_store) {  // the tensor stores complete before the CTA's shared memory is released
            bulk_wait_all();
            __syncwarp();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ CTA pairs (cta_group::2): 256 x BN output tiles
//
// A cluster of two CTAs on two SMs computes one 256 x BN output tile (BN 128, 192 or 256): CTA r loads rows
// m0 + 128 r of x and rows n0 + (BN / 2) r of W (its half of the tile's W columns) into its own shared memory, and
// CTA 0's single MMA thread issues tcgen05.mma.cta_group::2 (M 256, N BN, K 16), which reads both CTAs' halves and
// writes each CTA's 128 output rows (all BN columns) into that CTA's tensor memory. Per SM and K step the tensor cores
// then do 128 x BN x 64 products on 16 KB + BN x 64 B of shared-memory traffic (at BN 256: 128 FLOP a byte; the
// one-CTA 128 x 256 tile does 85), which is what the L2 feed allows at full tensor rate. Both CTAs' copies complete on
// CTA 0's full barrier (the barrier's address with the peer bit cleared); the MMA's commits arrive on both CTAs'
// barriers (tcgen05.commit multicast); each CTA's epilogue reads its own accumulator and releases it on CTA 0's
// barrier. No copy is broadcast: each CTA loads its own tiles.
template <int BN> struct PairCfg {
    static constexpr uint32_t STAGE = kABytes + uint32_t(BN / 2) * kBK * 2;  // x [128][64] + W half [BN / 2][64]
    static constexpr int STAGES = BN == 256 ? 6 : 7;
    static constexpr uint32_t SWB = BN == 128 ? 8192 : 4096;  // epilogue staging bytes a warp
    static constexpr uint32_t ACC = BN == 192 ? 256 : BN;                    // column offset of the second accumulator
    static constexpr uint32_t TMEM_COLS = 2 * ACC;                           // two accumulators (a power of two)
    static constexpr size_t SMEM = size_t(STAGES) * STAGE + 1024 + 256 + 4 * SWB + 4 * 1024;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of `p` (this CTA's shared memory) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(const void *p, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_addr(p)), "r"(rank));
    return d;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// One stage's copies of a pair CTA, issued by a whole converged warp through one elected lane: CTA 0's lane arrives
// on its full barrier expecting both CTAs' bytes; each CTA's two copies complete on CTA 0's barrier.
__device__ __forceinline__ void tma_stage_pair_warp(uint64_t *bar, bool leader, uint32_t bytes, uint32_t dst_a, const CUtensorMap *ma, int xa, int ya,
                                                    int za, uint32_t dst_b, const CUtensorMap *mb, int xb, int yb, int zb) {
    const uint32_t b = smem_addr(bar), b0 = b & 0xFEFFFFFFu;
    asm volatile("{\n\t.reg .pred e, l;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.and.b32 l, %13, 0, e;\n\t"
                 "@l mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t"
                 "@e cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%3, {%4, %5, %6}], [%12];\n\t"
                 "@e cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%7], [%8, {%9, %10, %11}], [%12];\n\t}"
                 ::"r"(b), "r"(bytes), "r"(dst_a), "l"(ma), "r"(xa), "r"(ya), "r"(za), "r"(dst_b), "l"(mb), "r"(xb), "r"(yb), "r"(zb), "r"(b0),
                 "r"(uint32_t(leader))
                 : "memory");
}
// tcgen05.mma.cta_group::2 issued by a whole converged warp, one lane elected (as umma_bf16_warp).
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on `bar` in both CTAs of the pair when every MMA the elected lane issued before has completed (whole warp).
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
    asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
                 "h"(uint16_t(3))
                 : "memory");
}

template <int BN, int EPI, bool F16 = false>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc2_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                                                                   const __grid_constant__ CUtensorMap ty, const GemmArgs g) {
    using P = PairCfg<BN>;
    constexpr int kPairStages = P::STAGES;
    constexpr uint32_t kPairStage = P::STAGE;
    constexpr uint32_t kIdesc = F16 ? umma_idesc_f16(256, BN) : umma_idesc_bf16(256, BN);
    extern __shared__ uint8_t gemm2_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gemm2_smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t s0 = smem_addr(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kPairStages * kPairStage + 4 * P::SWB);
    uint64_t *empty = full + kPairStages;
    uint64_t *tfull = empty + kPairStages;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(drain + 1);
    const uint32_t STG_BASE = s0 + kPairStages * kPairStage;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int mt = (g.M + 255) / 256, nt = (g.N + BN - 1) / BN;
    const int tiles = mt * nt * g.batches * g.groups, kt = (g.K + kBK - 1) / kBK;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&tfull[0], 1);
        mbar_init(&tfull[1], 1);
        mbar_init(&tempty[0], 8);  // four epilogue warps in each CTA (used on CTA 0)
        mbar_init(&tempty[1], 8);
        mbar_init(drain, 1);
        mbar_init_fence();
        tma_prefetch_desc(&ta);
        tma_prefetch_desc(&tb);
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tslot)), "r"(P::TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised and tensor memory allocated before any cross-CTA traffic
    tc_fence_after();
    pdl_enter();
    const uint32_t tmem = *tslot;
    bool ok = true;

    if (warp == 0) {
        // ---- tensor copies: this CTA's x rows and W half, completing on CTA 0's full barrier
        uint32_t it = 0;
        for (int t = pair; t < tiles && ok; t += npairs) {
            const int mi = t % mt, rest = t / mt, ni = rest % nt, z = rest / nt, zg = z % g.groups;
            for (int kc = 0; kc < kt; ++kc, ++it) {
                const int s = int(it % kPairStages);
                const uint32_t u = it / kPairStages;
                if (!mbar_wait_warp(&empty[s], (u & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t sa = s0 + uint32_t(s) * kPairStage;
                tma_stage_pair_warp(&full[s], leader, 2 * kPairStage, sa, &ta, kc * kBK, mi * 256 + 128 * int(rank), z, sa + kABytes, &tb, kc * kBK,
                                    ni * BN + (BN / 2) * int(rank), zg);
                __syncwarp();
            }
        }
        if (!ok && leader) {
            const uint32_t last = it;
            for (uint32_t j = last > uint32_t(kPairStages) ? last - kPairStages : 0; j < last; ++j)
                mbar_wait_warp(&full[j % kPairStages], (j / kPairStages) & 1u);
        }
    } else if (warp == 1) {
        // ---- MMA issue (CTA 0 only)
        if (leader) {
            uint32_t it = 0, tc = 0;
            for (int t = pair; t < tiles && ok; t += npairs, ++tc) {
                const uint32_t a = tc & 1u, v = tc >> 1;
                if (!mbar_wait_warp(&tempty[a], (v & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t dcol = tmem + a * P::ACC;
                for (int kc = 0; kc < kt; ++kc, ++it) {
                    const int s = int(it % kPairStages);
                    const uint32_t u = it / kPairStages;
                    if (!mbar_wait_warp(&full[s], u & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    {
                        const uint32_t sa = s0 + uint32_t(s) * kPairStage, sb = sa + kABytes;
#pragma unroll
                        for (int k = 0; k < kBK / 16; ++k)
                            umma_bf16_pair(dcol, umma_desc(sa + 32 * k, 16, 1024), umma_desc(sb + 32 * k, 16, 1024), kIdesc, (kc | k) != 0);
                        umma_commit_pair(&empty[s]);  // both CTAs' stage s is free once these MMAs have read it
                    }
                    __syncwarp();
                }
                if (!ok) break;
                umma_commit_pair(&tfull[a]);
                __syncwarp();
            }
            if (!ok) {
                umma_commit_pair(drain);
                __syncwarp();
                mbar_wait_warp(drain, 0);
            }
        }
    } else {
        // ---- epilogue: this CTA's 128 rows of the 256-row tile, all 256 columns
        const int q = warp & 3;
        const uint32_t stg = STG_BASE + uint32_t(warp - 2) * P::SWB;
        uint32_t seq = 0;
        const uint32_t tempty0 = map_rank(&tempty[0], 0);
        float *bias_s = reinterpret_cast<float *>(smem + kPairStages * kPairStage + 4 * P::SWB + 256) + (warp - 2) * 256;
        uint32_t tc = 0;
        for (int t = pair; t < tiles && ok; t += npairs, ++tc) {
            const uint32_t a = tc & 1u, v = tc >> 1;
            const int mi = t % mt, rest = t / mt, ni = rest % nt, z = rest / nt, zb = z / g.groups, zg = z % g.groups;
            EpiPre pre;
            epi_prepare<EPI>(g, ni * BN, BN, zg, mi * 256 + 128 * int(rank) + 32 * q + lane, lane, bias_s, pre);
            if (!mbar_wait_warp(&tfull[a], v & 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int n0 = ni * BN, nch = min(BN, g.N - n0 + 31) / 32;
            epilogue_tile<EPI, P::SWB>(g, &ty, tmem + (uint32_t(32 * q) << 16) + a * P::ACC, nch, mi * 256 + 128 * int(rank) + 32 * q, lane, n0, zb,
                                       zg, stg, seq, pre);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tempty0 + a * 8);
        }
        if (g.tma_store) {
            bulk_wait_all();
            __syncwarp();
        }
    }
    tc_fence_before();
    cluster_sync();  // the peer's last remote arrivals and reads are done before either CTA releases its memory
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------ quantized prefill GEMM (Q8 / Q4 weights)
//
// y[M][N] (+)= bias + x[M][K] . W[N][K]^T with W = code * scale[n][k / 32] (Vox's Q8 / Q4 blocks) and f32 x, on the
// tensor cores in f16 (kind::f16, f16 A and B, f32 accumulation). From 256 rows of x the product runs in two passes
// instead (gemm_q: q_w_to_f16_kernel, then the tcgen05 GEMM above on f16 operands; 70.4 / 67.5 us at 512 x 12288 x
// 4096 against 90.4 / 79.3 us in one pass), since here every CTA converts its weight tile once per 128 x rows. x is rounded to f16 once, by a small kernel before
// the GEMM (q_x_to_f16_kernel); the codes are converted inside the GEMM. Tile 128 activation rows x 256 weight rows,
// K step 64, one ring of three stages, each holding the x tile (f16, loaded by TMA straight into the 128-byte-swizzled
// MMA operand layout), the raw codes and the converted weight tile. Fourteen warps:
//   warp 0       TMA: a stage's x tile [128][64] f16 and codes [256][64] bytes (Q8) or [256][32] (Q4);
//   warps 6..13  converters: codes to f16 by the exponent trick (0x6400 | u is 1024 + u exactly; minus the code offset
//                gives the integer code, times the block's scale rounds once to f16), written as the 128-byte-swizzled
//                K-major weight tile of the same stage;
//   warp 1       issues tcgen05.mma (M 128, N 256, K 16) through an elected lane into one of two TMEM accumulators
//                (512 columns) and frees the stage when its MMAs have read it;
//   warps 2..5   the epilogue (bias, accumulate, f32 store) as in the bf16 GEMM.
// Measured at 512 x 12288 x 4096 (Q8 / Q4): converting x inside the GEMM (an f32 raw ring beside the f16 one, two
// stages each) took 144 / 141 us; this ring 118 / 98 us. Not kept: a separate code ring loaded up to three steps ahead
// with the x copies started by the converters (122 / 115 us), and the next step's block scales loaded while the
// current one converts (142 / 132 us). With the last wave split into K-ranges (q_item, gemm_q_fixup_kernel): 90.0 /
// 79.1 us; not kept there: CTA pairs on 256 x 256 tiles (cta_group::2, each CTA converting 128 weight rows: 131 / 127
// us) and the block scales loaded one K step ahead (99 / 88 us). f16 keeps 11 significant bits of x and of code *
// scale (bf16: 8); |x| must stay below 65504. A code's integer value is exact in f16; its product with an f16 scale is
// rounded once.
constexpr int kQBN = 256;
constexpr int kQThreads = 448;
constexpr int kQConvWarps = 8;
constexpr uint32_t kQA = kBM * kBK * 2;             // x tile, 16 KB f16
constexpr uint32_t kQB = kQBN * kBK * 2;            // weight tile, 32 KB f16
template <bool Q4> struct QCfg {
    static constexpr uint32_t CODES = Q4 ? kQBN * kBK / 2 : kQBN * kBK;  // raw code bytes a K step
    static constexpr uint32_t STAGE = kQA + kQB + CODES;                 // 64 KB (Q8), 56 KB (Q4); multiples of 1024
    static constexpr int S = 3;
    static constexpr size_t SMEM = size_t(S) * STAGE + 1024 + 256 + 4 * 4096 + 4 * 1024;
};

// Two codes (bytes b0, b1 of w, already offset to unsigned) as f16x2 1024 + u: prmt puts the code byte under 0x64.
__device__ __forceinline__ uint32_t f16_pair_1024(uint32_t w, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(w), "r"(0x64646464u), "r"(sel));
    return d;
}
__device__ __forceinline__ uint32_t hsub_hmul(uint32_t v, uint32_t off2, uint32_t s2) {
    uint32_t d;
    asm("{\n\t.reg .b32 t;\n\tsub.rn.f16x2 t, %1, %2;\n\tmul.rn.f16x2 %0, t, %3;\n\t}" : "=r"(d) : "r"(v), "r"(off2), "r"(s2));
    return d;
}
__device__ __forceinline__ uint32_t f16x2_of(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// xh = f16(x) (round to nearest), four elements a thread and pass (n a multiple of 4; x and xh 16- and 8-byte aligned).
__global__ void __launch_bounds__(256) q_x_to_f16_kernel(const float4 *x, uint2 *xh, int64_t n4) {
    pdl_enter();
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
        const float4 v = __ldg(x + i);
        xh[i] = make_uint2(f16x2_of(v.x, v.y), f16x2_of(v.z, v.w));
    }
}

// The two-pass form's weight pass: w16[e] = f16(code(e)) * f16(scale[e / 32]) for the flat element e of W [N][K]
// (K a multiple of 32, so a 32-block is the flat e / 32), with the converters' arithmetic of gemm_q_kernel (the code
// exact in f16 by the 0x64 exponent pattern, one rounding of the product): the f16 operands are the same either way.
// Eight weights a thread and pass: Q8 bytes e .. e + 7; Q4 the low (e % 32 < 16) or high nibbles of the block's bytes
// (e % 16) .. (e % 16) + 7 (Vox's order: byte j holds elements j and j + 16).
template <bool Q4, bool SF16>
__global__ void __launch_bounds__(256) q_w_to_f16_kernel(const uint8_t *w, const void *scale, uint4 *w16, int64_t n8) {
    pdl_enter();
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t e = 8 * i, blk = e >> 5;
        const float sc = SF16 ? __half2float(__ldg(reinterpret_cast<const __half *>(scale) + blk)) : __ldg(reinterpret_cast<const float *>(scale) + blk);
        const __half h = __float2half_rn(sc);
        const uint32_t hb = *reinterpret_cast<const uint16_t *>(&h), s2 = hb | (hb << 16);
        uint32_t c[2], off;
        if constexpr (Q4) {
            const int p = int(e & 31);
            const uint2 v = __ldg(reinterpret_cast<const uint2 *>(w + blk * 16 + (p & 15)));
            const int sh = p < 16 ? 0 : 4;
            c[0] = (v.x >> sh) & 0x0F0F0F0Fu, c[1] = (v.y >> sh) & 0x0F0F0F0Fu;
            off = 0x64086408u;  // f16x2 (1032, 1032): 1024 + 8
        } else {
            const uint2 v = __ldg(reinterpret_cast<const uint2 *>(w + e));
            c[0] = v.x ^ 0x80808080u, c[1] = v.y ^ 0x80808080u;
            off = 0x64806480u;  // f16x2 (1152, 1152): 1024 + 128
        }
        uint4 o;
        o.x = hsub_hmul(f16_pair_1024(c[0], 0x4140u), off, s2);
        o.y = hsub_hmul(f16_pair_1024(c[0], 0x4342u), off, s2);
        o.z = hsub_hmul(f16_pair_1024(c[1], 0x4140u), off, s2);
        o.w = hsub_hmul(f16_pair_1024(c[1], 0x4342u), off, s2);
        w16[i] = o;
    }
}

struct GemmQArgs {
    int M, N, K, nblk;      // nblk = K / 32
    const void *scale;      // [N][nblk] f32 or f16
    GemmArgs g;             // epilogue (kEpiF32: bias, accumulate, y [M][N])
    // Work items (one CTA takes items blockIdx.x, + gridDim.x, ...): items 0 .. full - 1 are whole output tiles, the
    // rest are `splits` K-ranges of each of the last `rem` tiles (piece p of tail tile i is item full + p * rem + i),
    // whose f32 partials go to part[item - full][128][256] and are summed in piece order by gemm_q_fixup_kernel.
    int full, rem, splits, items;
    float *part;
};

// Tile, K-step range and partial slot (-1: the whole tile, finished into y) of work item w.
struct QItem {
    int t, kb, ke, slot;
};
__device__ __forceinline__ QItem q_item(const GemmQArgs &q, int w, int kt) {
    QItem r;
    if (w < q.full) {
        r.t = w, r.kb = 0, r.ke = kt, r.slot = -1;
        return r;
    }
    const int j = w - q.full, p = j / q.rem;
    r.t = q.full + (j - p * q.rem), r.slot = j;
    r.kb = int(int64_t(p) * kt / q.splits), r.ke = int(int64_t(p + 1) * kt / q.splits);  // splits <= kt: never empty
    return r;
}

template <bool Q4, bool SF16>
__global__ void __launch_bounds__(kQThreads, 1) gemm_q_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                                                              const GemmQArgs q) {
    using C = QCfg<Q4>;
    constexpr uint32_t kIdesc = (1u << 4) | (uint32_t(kQBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);  // f16 A and B, f32 D
    extern __shared__ uint8_t gq_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gq_smem_raw) + 1023) & ~uintptr_t(1023));
    // stages [S][x f16 (A) | weights f16 (B) | codes], 1024-aligned; then the barriers, staging and bias slots
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(smem + C::S * C::STAGE);  // x and codes landed (TMA)
    uint64_t *conv_full = raw_full + C::S;                                      // weights converted (8 warps)
    uint64_t *stage_empty = conv_full + C::S;                                   // the stage's MMAs have completed
    uint64_t *tfull = stage_empty + C::S;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(drain + 1);
    const uint32_t STG_BASE = smem_addr(smem + C::S * C::STAGE) + 256;  // the epilogue warps' staging areas (after the barriers)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (q.M + kBM - 1) / kBM, kt = (q.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&conv_full[s], kQConvWarps);
            mbar_init(&stage_empty[s], 1);
        }
        mbar_init(&tfull[0], 1);
        mbar_init(&tfull[1], 1);
        mbar_init(&tempty[0], 4);
        mbar_init(&tempty[1], 4);
        mbar_init(drain, 1);
        mbar_init_fence();
        tma_prefetch_desc(&tx);
        tma_prefetch_desc(&tw);
    }
    if (warp == 0) tmem_alloc(tslot, 2 * kQBN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_enter();
    const uint32_t tmem = *tslot;
    bool ok = true;

    if (warp == 0) {
        // ---- copies: a stage's x tile (into its MMA operand slot) and codes
        uint32_t it = 0;
        for (int w = blockIdx.x; w < q.items && ok; w += gridDim.x) {
            const QItem wi = q_item(q, w, kt);
            const int m0 = (wi.t % mt) * kBM, n0 = (wi.t / mt) * kQBN;
            for (int kc = wi.kb; kc < wi.ke; ++kc, ++it) {
                const int s = int(it % C::S);
                const uint32_t u = it / C::S;
                if (!mbar_wait_warp(&stage_empty[s], (u & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t sa = smem_addr(smem + s * C::STAGE);
                tma_stage_warp(&raw_full[s], kQA + C::CODES, sa, &tx, kc * kBK, m0, 0, sa + kQA + kQB, &tw, kc * (Q4 ? kBK / 2 : kBK), n0, 0);
                __syncwarp();
            }
        }
        if (!ok) {
            const uint32_t last = it;
            for (uint32_t j = last > uint32_t(C::S) ? last - C::S : 0; j < last; ++j) mbar_wait_warp(&raw_full[j % C::S], (j / C::S) & 1u);
        }
    } else if (warp >= 6) {
        // ---- converters: thread ct of 256
        const int ct = threadIdx.x - 6 * 32;
        uint32_t it = 0;
        const uint32_t off8 = 0x64806480u;   // f16x2 (1152, 1152): 1024 + 128 (Q8 codes offset to unsigned by ^ 0x80)
        const uint32_t off4 = 0x64086408u;   // f16x2 (1032, 1032): 1024 + 8 (Q4 codes are u - 8)
        for (int w = blockIdx.x; w < q.items && ok; w += gridDim.x) {
            const QItem wi = q_item(q, w, kt);
            const int n0 = (wi.t / mt) * kQBN;
            for (int kc = wi.kb; kc < wi.ke; ++kc, ++it) {
                const int rs = int(it % C::S);
                const uint32_t ru = it / C::S;
                // the block scales of this thread's weight tasks (global loads, in flight during the waits)
                constexpr int NT = Q4 ? 2 : 4;  // weight tasks a thread
                uint32_t s2[NT];
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const int i = ct + 256 * j;
                    const int row = Q4 ? i >> 1 : i >> 2, blk = kc * 2 + (Q4 ? (i & 1) : ((i & 3) >> 1));
                    float sc = 0.f;
                    if (n0 + row < q.N && blk < q.nblk) {
                        const int64_t e = int64_t(n0 + row) * q.nblk + blk;
                        sc = SF16 ? __half2float(__ldg(reinterpret_cast<const __half *>(q.scale) + e)) : __ldg(reinterpret_cast<const float *>(q.scale) + e);
                    }
                    const __half h = __float2half_rn(sc);
                    const uint32_t hb = *reinterpret_cast<const uint16_t *>(&h);
                    s2[j] = hb | (hb << 16);
                }
                // the stage was reloaded only after its previous MMAs completed, so its weight tile is free
                if (!mbar_wait_warp(&raw_full[rs], ru & 1u)) {
                    ok = false;
                    break;
                }
                const uint8_t *sp = smem + rs * C::STAGE;
                const uint32_t cb = smem_addr(sp) + kQA;
                const uint8_t *rc = sp + kQA + kQB;
                if constexpr (!Q4) {
                    // 16 codes a task: row i / 4, 16-code quarter i % 4 (block quarter / 2)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int i = ct + 256 * j, row = i >> 2, qq = i & 3;
                        const uint4 w = *reinterpret_cast<const uint4 *>(rc + i * 16);
                        const uint32_t ws[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
                        uint32_t h[8];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            h[2 * k] = hsub_hmul(f16_pair_1024(ws[k], 0x4140u), off8, s2[j]);
                            h[2 * k + 1] = hsub_hmul(f16_pair_1024(ws[k], 0x4342u), off8, s2[j]);
                        }
                        const uint32_t b0 = cb + row * 128;
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b0 + ((((2 * qq) ^ (row & 7))) << 4)), "r"(h[0]), "r"(h[1]),
                                     "r"(h[2]), "r"(h[3]) : "memory");
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b0 + ((((2 * qq + 1) ^ (row & 7))) << 4)), "r"(h[4]),
                                     "r"(h[5]), "r"(h[6]), "r"(h[7]) : "memory");
                    }
                } else {
                    // one 16-byte block a task (32 codes): row i / 2, block i % 2; byte j: code j (low), j + 16 (high)
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int i = ct + 256 * j, row = i >> 1, bb = i & 1;
                        const uint4 w = *reinterpret_cast<const uint4 *>(rc + i * 16);
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
                        uint32_t lo[8], hi[8];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t l = ws[k] & 0x0F0F0F0Fu, hh = (ws[k] >> 4) & 0x0F0F0F0Fu;
                            lo[2 * k] = hsub_hmul(f16_pair_1024(l, 0x4140u), off4, s2[j]);
                            lo[2 * k + 1] = hsub_hmul(f16_pair_1024(l, 0x4342u), off4, s2[j]);
                            hi[2 * k] = hsub_hmul(f16_pair_1024(hh, 0x4140u), off4, s2[j]);
                            hi[2 * k + 1] = hsub_hmul(f16_pair_1024(hh, 0x4342u), off4, s2[j]);
                        }
                        const uint32_t b0 = cb + row * 128;
                        const int c0 = 4 * bb;  // the block's 32 elements: chunks 4 bb .. 4 bb + 3
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b0 + (((c0 + 0) ^ (row & 7)) << 4)), "r"(lo[0]), "r"(lo[1]),
                                     "r"(lo[2]), "r"(lo[3]) : "memory");
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b0 + (((c0 + 1) ^ (row & 7)) << 4)), "r"(lo[4]), "r"(lo[5]),
                                     "r"(lo[6]), "r"(lo[7]) : "memory");
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b0 + (((c0 + 2) ^ (row & 7)) << 4)), "r"(hi[0]), "r"(hi[1]),
                                     "r"(hi[2]), "r"(hi[3]) : "memory");
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b0 + (((c0 + 3) ^ (row & 7)) << 4)), "r"(hi[4]), "r"(hi[5]),
                                     "r"(hi[6]), "r"(hi[7]) : "memory");
                    }
                }
                fence_proxy_async();  // the generic-proxy writes, visible to the MMA (async proxy)
                __syncwarp();
                if (lane == 0) mbar_arrive(&conv_full[rs]);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue
        uint32_t it = 0, tc = 0;
        for (int w = blockIdx.x; w < q.items && ok; w += gridDim.x, ++tc) {
            const QItem wi = q_item(q, w, kt);
            const uint32_t a = tc & 1u, v = tc >> 1;
            if (!mbar_wait_warp(&tempty[a], (v & 1u) ^ 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t dcol = tmem + a * kQBN;
            for (int kc = wi.kb; kc < wi.ke; ++kc, ++it) {
                const int s = int(it % C::S);
                const uint32_t u = it / C::S;
                // the x tile (TMA) and the converted weights
                if (!mbar_wait_warp(&raw_full[s], u & 1u) || !mbar_wait_warp(&conv_full[s], u & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                {
                    const uint32_t sa = smem_addr(smem + s * C::STAGE), sb = sa + kQA;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        umma_bf16_warp(dcol, umma_desc(sa + 32 * k, 16, 1024), umma_desc(sb + 32 * k, 16, 1024), kIdesc, kc != wi.kb || k != 0);
                    umma_commit_warp(&stage_empty[s]);  // the stage returns to the copy warp when these MMAs have read it
                }
                __syncwarp();
            }
            if (!ok) break;
            umma_commit_warp(&tfull[a]);
            __syncwarp();
        }
        if (!ok) {
            umma_commit_warp(drain);
            __syncwarp();
            mbar_wait_warp(drain, 0);
        }
    } else {
        // ---- epilogue (warps 2..5)
        const int qw = warp & 3;
        const uint32_t stg = STG_BASE + uint32_t(warp - 2) * kStageWarpBytes;
        float *bias_s = reinterpret_cast<float *>(smem + C::S * C::STAGE + 256 + 4 * kStageWarpBytes) + (warp - 2) * 256;
        uint32_t qseq = 0;
        uint32_t tc = 0;
        for (int w = blockIdx.x; w < q.items && ok; w += gridDim.x, ++tc) {
            const QItem wi = q_item(q, w, kt);
            const uint32_t a = tc & 1u, v = tc >> 1;
            const int m0 = (wi.t % mt) * kBM, n0 = (wi.t / mt) * kQBN;
            // a K-range piece stores its raw f32 partial in its [128][256] slot (no bias, no accumulate): y is addressed
            // as slot - (m0 row pitch + n0) so that the epilogue's absolute rows and columns land inside the slot
            GemmArgs ga = q.g;
            if (wi.slot >= 0) {
                ga.bias = nullptr, ga.accumulate = 0, ga.ldy = kQBN;
                ga.y = reinterpret_cast<void *>(reinterpret_cast<uintptr_t>(q.part) +
                                                uintptr_t((int64_t(wi.slot) * kBM * kQBN - int64_t(m0) * kQBN - n0) * int64_t(sizeof(float))));
            }
            EpiPre pre;
            epi_prepare<kEpiF32>(ga, n0, kQBN, 0, m0 + 32 * qw + lane, lane, bias_s, pre);
            if (!mbar_wait_warp(&tfull[a], v & 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int nch = min(kQBN, q.N - n0 + 31) / 32;
            epilogue_tile<kEpiF32, kStageWarpBytes>(ga, nullptr, tmem + (uint32_t(32 * qw) << 16) + a * kQBN, nch, m0 + 32 * qw, lane, n0, 0, 0, stg,
                                                    qseq, pre);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * kQBN);
    }
}

// The tail tiles of a split schedule: y = (sum of the tile's K-range partials, in piece order) + bias (+ y), each element
// added in the order the whole-tile epilogue uses, so the result is the same run to run. Four columns a thread.
__global__ void __launch_bounds__(256) gemm_q_fixup_kernel(const GemmQArgs q) {
    pdl_enter();
    constexpr int kQuads = kBM * kQBN / 4;
    const int mt = (q.M + kBM - 1) / kBM;
    const size_t slot = size_t(q.rem) * kBM * kQBN;  // floats between piece p and piece p + 1 of one tile
    const int64_t total = int64_t(q.rem) * kQuads;
    float *y = reinterpret_cast<float *>(q.g.y);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int ti = int(i / kQuads), e = int(i - int64_t(ti) * kQuads);
        const int r = e / (kQBN / 4), c = (e % (kQBN / 4)) * 4;
        const int t = q.full + ti;
        const int gm = (t % mt) * kBM + r, gn = (t / mt) * kQBN + c;
        if (gm >= q.M || gn >= q.N) continue;
        const float *pp = q.part + size_t(ti) * kBM * kQBN + size_t(r) * kQBN + c;
        float4 a = *reinterpret_cast<const float4 *>(pp);
        for (int p = 1; p < q.splits; ++p) {
            const float4 b = *reinterpret_cast<const float4 *>(pp + p * slot);
            a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
        }
        const float v[4] = {a.x, a.y, a.z, a.w};
        float *yr = y + int64_t(gm) * q.g.ldy + gn;
        const int nv = min(4, q.N - gn);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j >= nv) break;
            float f = v[j];
            if (q.g.bias) f += __ldg(q.g.bias + gn + j);
            yr[j] = q.g.accumulate ? f + yr[j] : f;
        }
    }
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// 3-D bf16 (or f16: dt) map of planes [depth][rows][cols] (row pitch ld elements, plane pitch rows * ld), box 64 x
// box_rows x 1, 128-byte swizzle, zero fill past every edge.
int bf16_map(const void *base, int64_t cols, int64_t rows, int64_t depth, int64_t ld, int box_rows, CUtensorMap &m, const char *name,
             CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
    auto fn = encode();
    if (!fn) return set_error(VOX_CUDA_ERR_DEVICE, std::string(name) + ": cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(depth)};
    const cuuint64_t strides[2] = {cuuint64_t(ld) * 2, cuuint64_t(ld) * 2 * cuuint64_t(rows)};
    const cuuint32_t box[3] = {uint32_t(kBK), uint32_t(box_rows), 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(&m, dt, 3, const_cast<void *>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VOX_CUDA_ERR_ARG, std::string(name) + ": tensor map rejected (code " + std::to_string(int(r)) + ")");
    return VOX_CUDA_OK;
}

// 3-D map (depth 1) of a row-major [rows][cols] matrix of 1- or 4-byte elements, row pitch ld_bytes, box box_cols x
// box_rows, no swizzle, zero fill past the edges.
int plain_map(const void *base, CUtensorMapDataType dt, int64_t cols, int64_t rows, int64_t ld_bytes, int box_cols, int box_rows,
              CUtensorMap &m, const char *name) {
    auto fn = encode();
    if (!fn) return set_error(VOX_CUDA_ERR_DEVICE, std::string(name) + ": cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), 1};
    const cuuint64_t strides[2] = {cuuint64_t(ld_bytes), cuuint64_t(ld_bytes) * cuuint64_t(rows)};
    const cuuint32_t box[3] = {uint32_t(box_cols), uint32_t(box_rows), 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(&m, dt, 3, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VOX_CUDA_ERR_ARG, std::string(name) + ": tensor map rejected (code " + std::to_string(int(r)) + ")");
    return VOX_CUDA_OK;
}

// 3-D map of the GEMM output y: planes [depth][rows][cols] of f32 or bf16 (row pitch ld_bytes, plane pitch
// plane_bytes), box 32 x 32 x 1 in the swizzle the epilogue stages with (128-byte rows: 128-byte swizzle; 64-byte
// rows: 64-byte swizzle).
int y_map(const void *base, bool f32, int64_t cols, int64_t rows, int64_t depth, int64_t ld_bytes, int64_t plane_bytes, CUtensorMap &m,
          const char *name) {
    auto fn = encode();
    if (!fn) return set_error(VOX_CUDA_ERR_DEVICE, std::string(name) + ": cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(depth)};
    const cuuint64_t strides[2] = {cuuint64_t(ld_bytes), cuuint64_t(plane_bytes)};
    const cuuint32_t box[3] = {32, 32, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides,
                          box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VOX_CUDA_ERR_ARG, std::string(name) + ": output tensor map rejected (code " + std::to_string(int(r)) + ")");
    return VOX_CUDA_OK;
}

template <bool Q4, bool SF16>
int launch_q(const CUtensorMap &tx, const CUtensorMap &tw, const GemmQArgs &q, cudaStream_t st, const char *name) {
    auto kern = gemm_q_kernel<Q4, SF16>;
    static bool attr_set[128] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 128 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(QCfg<Q4>::SMEM)) != cudaSuccess) return check_launch(name);
        attr_set[dev] = true;
    }
    const int grid = q.items < sm_count() ? q.items : sm_count();
    launch_k(kern, grid, kQThreads, QCfg<Q4>::SMEM, st, tx, tw, q);
    int rc = check_launch(name);
    if (rc == VOX_CUDA_OK && q.splits > 1) {
        launch_k(gemm_q_fixup_kernel, grid_for(int64_t(q.rem) * kBM * kQBN / 4, 256, 8), 256, 0, st, q);
        rc = check_launch(name);
    }
    return rc;
}

template <int BN, int EPI, bool F16 = false>
int launch(const GemmPlan &p, cudaStream_t st, const char *name) {
    auto kern = gemm_tc_kernel<BN, EPI, F16>;
    static bool attr_set[128] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 128 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg<BN>::SMEM)) != cudaSuccess) return check_launch(name);
        attr_set[dev] = true;
    }
    const int mt = (p.a.M + kBM - 1) / kBM, nt = (p.a.N + BN - 1) / BN;
    const int64_t tiles = int64_t(mt) * nt * p.a.batches * p.a.groups;
    const int grid = int(tiles < sm_count() ? tiles : sm_count());
    launch_k(kern, grid, kGemmThreads, Cfg<BN>::SMEM, st, p.ta, p.tb, p.ty, p.a);
    return check_launch(name);
}

template <int BN, int EPI, bool F16 = false>
int launch_pair(const GemmPlan &p, cudaStream_t st, const char *name) {
    auto kern = gemm_tc2_kernel<BN, EPI, F16>;
    constexpr size_t kPairSmem = PairCfg<BN>::SMEM;
    static bool attr_set[128] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 128 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPairSmem)) != cudaSuccess) return check_launch(name);
        attr_set[dev] = true;
    }
    const int64_t tiles = int64_t((p.a.M + 255) / 256) * ((p.a.N + BN - 1) / BN) * p.a.batches * p.a.groups;
    const int64_t pairs = sm_count() / 2;
    const int grid = 2 * int(tiles < pairs ? tiles : pairs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = kPairSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    if (cudaLaunchKernelEx(&cfg, kern, p.ta, p.tb, p.ty, p.a) != cudaSuccess) return check_launch(name);
    return VOX_CUDA_OK;
}

template <int EPI, bool F16 = false>
int launch_bn(const GemmPlan &p, cudaStream_t st, const char *name) {
    if (p.pair) {
        if (p.bn == 128) return launch_pair<128, EPI, F16>(p, st, name);
        if (p.bn == 192) return launch_pair<192, EPI, F16>(p, st, name);
        return launch_pair<256, EPI, F16>(p, st, name);
    }
    if (p.bn == 64) return launch<64, EPI, F16>(p, st, name);
    if (p.bn == 256) return launch<256, EPI, F16>(p, st, name);
    return launch<128, EPI, F16>(p, st, name);
}

}  // namespace

int gemm_plan(const void *x, int64_t ldx, const void *w, int64_t ldw, const GemmArgs &a, int epi, GemmPlan &plan, const char *name) {
    VOX_REQUIRE(a.M > 0 && a.N > 0 && a.K > 0 && a.batches > 0 && a.groups > 0, std::string(name) + ": bad GEMM shape");
    VOX_REQUIRE(x && w && a.y, std::string(name) + ": NULL pointer");
    VOX_REQUIRE(a.K % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 && ldx >= a.K && ldw >= a.K && aligned16(x) && aligned16(w),
                std::string(name) + ": x and W need 16-byte aligned rows (K and the row pitches multiples of 8)");
    VOX_REQUIRE(epi >= kEpiF32 && epi <= kEpiGeluErfF32, std::string(name) + ": unknown epilogue");
    VOX_REQUIRE(!a.f16 || epi == kEpiF32, std::string(name) + ": f16 operands take the f32 epilogue only");
    if (epi == kEpiQkvRope)
        VOX_REQUIRE(a.cs && a.inner > 0 && a.inner % 64 == 0 && a.hd == 64 && a.N == 3 * a.inner && a.frames > 0,
                    std::string(name) + ": RoPE epilogue needs heads of 64 and 3 inner columns");
    plan.a = a;
    plan.epi = epi;
    // Tile shape: each candidate's time is estimated as waves x (K steps x t_step + t_wave) + t_fixed (+ t_f32 for an
    // f32 output), with waves = ceil(tiles / CTAs that fit: the SM count, or half of it for pairs), and the cheapest is
    // taken. The constants (us) are least-squares fits of measured launches on B200 (F5-base projections, a
    // 512 x 12288 x 4096 prefill GEMM; bf16 and f32 outputs): a K step of 64 costs 0.26 us on 128 x 128 tiles (the
    // copy and MMA issue rate), 0.40 us on 128 x 256 (the tensor cores); pairs halve the W bytes per CTA but pay a
    // larger fixed cost (cluster launch and first copies). The 128 x 64 tile's constants are scaled from the 128 x 128
    // tile's. VOX_CUDA_GEMM_BN (64 / 128 / 192 / 256) and VOX_CUDA_GEMM_PAIR (0 / 1) restrict the candidates (for
    // comparisons and tests; read at every plan).
    const int64_t sms = sm_count(), z = int64_t(a.batches) * a.groups, kt = (a.K + kBK - 1) / kBK;
    const char *ebn = std::getenv("VOX_CUDA_GEMM_BN"), *epair = std::getenv("VOX_CUDA_GEMM_PAIR");
    const int fv = ebn ? std::atoi(ebn) : 0;
    const int forced = fv == 64 || fv == 128 || fv == 192 || fv == 256 ? fv : 0;
    const int pair_mode = epair && epair[0] == '0' ? 0 : epair && epair[0] == '1' ? 1 : -1;
    const bool f32y = epi == kEpiF32 || epi == kEpiGeluTanhF32 || epi == kEpiGeluErfF32;
    struct Cand {
        bool pair;
        int bn;
        double step, wave, fixed, f32;
    };
    static constexpr Cand kCands[] = {{false, 64, 0.20, 0.20, 1.9, 0.6},   {false, 128, 0.261, 0.275, 2.0, 1.12},
                                      {false, 256, 0.395, 0.856, 2.46, 1.77}, {true, 128, 0.225, 0.542, 4.9, 0.81},
                                      {true, 192, 0.275, 1.473, 3.43, 1.29},  {true, 256, 0.316, 0.717, 5.56, 1.41}};
    double best = -1;
    for (const Cand &c : kCands) {
        if ((forced && c.bn != forced) || (pair_mode >= 0 && c.pair != (pair_mode == 1))) continue;
        if (a.tile && (c.bn != a.tile % 1000 || c.pair != (a.tile >= 1000))) continue;
        const int64_t units = ((a.M + (c.pair ? 255 : 127)) / (c.pair ? 256 : 128)) * ((a.N + c.bn - 1) / c.bn) * z;
        const int64_t slots = c.pair ? sms / 2 : sms, waves = (units + slots - 1) / slots;
        const double cost = double(waves) * (double(kt) * c.step + c.wave) + c.fixed + (f32y ? c.f32 : 0.0);
        if (best < 0 || cost < best) best = cost, plan.pair = c.pair, plan.bn = c.bn;
    }
    if (best < 0) plan.pair = forced == 192, plan.bn = forced ? forced : 128;  // contradictory overrides
    // x boxes of 128 rows; W boxes of BN rows (one CTA) or BN / 2 (each CTA of a pair)
    const CUtensorMapDataType odt = a.f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    int rc = bf16_map(x, a.K, a.M, z, ldx, kBM, plan.ta, name, odt);
    if (rc != VOX_CUDA_OK) return rc;
    rc = bf16_map(w, a.K, a.N, a.groups, ldw, plan.pair ? plan.bn / 2 : plan.bn, plan.tb, name, odt);
    if (rc != VOX_CUDA_OK) return rc;
    // y by tensor stores of 32 x 32 blocks where its layout allows: planes [batches][M][columns] with 16-byte aligned
    // rows, group g's columns at g * y_gstride (whole 32-column blocks, so no block of one group reaches the next);
    // otherwise by the threads' own stores. VOX_CUDA_GEMM_TMA_STORE=0 selects the latter (for comparisons).
    const bool f32out = epi == kEpiF32 || epi == kEpiGeluTanhF32 || epi == kEpiGeluErfF32;
    const int64_t es = f32out ? 4 : 2;
    const char *ets = std::getenv("VOX_CUDA_GEMM_TMA_STORE");
    const bool tma_ok = !(ets && ets[0] == '0') && aligned16(a.y) && (a.ldy * es) % 16 == 0 && a.ldy >= a.N &&
                        (a.batches == 1 || (a.y_bstride * es) % 16 == 0) &&
                        (a.groups == 1 || (a.N % 32 == 0 && (a.y_gstride * es) % 16 == 0)) && (!a.accumulate || f32out);
    const char *ewe = std::getenv("VOX_CUDA_GEMM_W_EARLY");  // 0: no early weight copies (for comparisons)
    if (ewe && ewe[0] == '0') plan.a.w_early = 0;
    plan.a.tma_store = 0;
    if (tma_ok) {
        const int64_t cols = int64_t(a.groups - 1) * a.y_gstride + a.N;
        const int64_t bstride = a.batches > 1 ? a.y_bstride : int64_t(a.M) * a.ldy;
        rc = y_map(a.y, f32out, cols, a.M, a.batches, a.ldy * es, bstride * es, plan.ty, name);
        if (rc != VOX_CUDA_OK) return rc;
        plan.a.tma_store = 1;
    }
    return VOX_CUDA_OK;
}

int gemm_run(const GemmPlan &p, cudaStream_t st, const char *name) {
    if (p.a.f16) return launch_bn<kEpiF32, true>(p, st, name);  // (gemm_plan admits f16 operands with kEpiF32 only)
    switch (p.epi) {
        case kEpiF32: return launch_bn<kEpiF32>(p, st, name);
        case kEpiBf16: return launch_bn<kEpiBf16>(p, st, name);
        case kEpiQkvRope: return launch_bn<kEpiQkvRope>(p, st, name);
        case kEpiGeluTanh: return launch_bn<kEpiGeluTanh>(p, st, name);
        case kEpiGeluErf: return launch_bn<kEpiGeluErf>(p, st, name);
        case kEpiGeluTanhF32: return launch_bn<kEpiGeluTanhF32>(p, st, name);
        default: return launch_bn<kEpiGeluErfF32>(p, st, name);
    }
}

// The quantized prefill GEMM: y[m][rows] (+)= bias + x[m][cols] . W^T with Q8 / Q4 weights (vox_cuda_gemm_q8 / q4).
int gemm_q(bool q4, const void *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y, int64_t rows,
           int64_t cols, int64_t m, int accumulate, cudaStream_t st, const char *name) {
    VOX_REQUIRE(scale_dtype == VOX_CUDA_F32 || scale_dtype == VOX_CUDA_F16, std::string(name) + ": scale dtype must be F32 or F16");
    VOX_REQUIRE(rows >= 0 && cols > 0 && m >= 0 && cols % 32 == 0, std::string(name) + ": bad shape (cols must be a multiple of 32)");
    VOX_REQUIRE(rows < (int64_t(1) << 31) && cols < (int64_t(1) << 31) && m < (int64_t(1) << 31), std::string(name) + ": shape too large");
    if (rows == 0 || m == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(w && scale && x && y, std::string(name) + ": NULL pointer");
    VOX_REQUIRE(aligned16(w) && aligned16(x), std::string(name) + ": w and x must be 16-byte aligned");
    GemmQArgs q{};
    q.M = int(m), q.N = int(rows), q.K = int(cols), q.nblk = int(cols / 32), q.scale = scale;
    q.g.M = int(m), q.g.N = int(rows), q.g.K = int(cols), q.g.y = y, q.g.ldy = rows, q.g.bias = bias, q.g.accumulate = accumulate != 0;
    // Two passes for prefill batches of 256 rows or more: W dequantised to f16 once (an HBM-bound pass of 3 bytes a Q8
    // weight), then the tcgen05 GEMM on f16 x and W, whose CTAs share converted weights through L2 instead of each
    // converting its tile (the one-pass kernel converts every weight tile once per 128 activation rows). The
    // operands are the one-pass kernel's, rounded the same way. VOX_CUDA_GEMMQ_TWOPASS=0 / 1 forces a form.
    bool two = m >= 256;
    if (const char *et = std::getenv("VOX_CUDA_GEMMQ_TWOPASS")) two = et[0] == '1';
    if (two) {
        void *buf = nullptr;
        const size_t xb = (size_t(m * cols * 2) + 255) & ~size_t(255), wb = size_t(rows) * size_t(cols) * 2;
        if (cudaMallocAsync(&buf, xb + wb, st) != cudaSuccess) return check_launch(name);
        void *xh = buf, *w16 = reinterpret_cast<uint8_t *>(buf) + xb;
        const int64_t n4 = m * cols / 4, n8 = rows * cols / 8;
        launch_k(q_x_to_f16_kernel, grid_for(n4, 256, 4), 256, 0, st, reinterpret_cast<const float4 *>(x), reinterpret_cast<uint2 *>(xh), n4);
        int rc = check_launch(name);
        if (rc == VOX_CUDA_OK) {
            const bool f16s = scale_dtype == VOX_CUDA_F16;
            const uint8_t *wu = reinterpret_cast<const uint8_t *>(w);
            uint4 *wo = reinterpret_cast<uint4 *>(w16);
            if (q4) {
                if (f16s) launch_k(q_w_to_f16_kernel<true, true>, grid_for(n8, 256, 8), 256, 0, st, wu, scale, wo, n8);
                else launch_k(q_w_to_f16_kernel<true, false>, grid_for(n8, 256, 8), 256, 0, st, wu, scale, wo, n8);
            } else {
                if (f16s) launch_k(q_w_to_f16_kernel<false, true>, grid_for(n8, 256, 8), 256, 0, st, wu, scale, wo, n8);
                else launch_k(q_w_to_f16_kernel<false, false>, grid_for(n8, 256, 8), 256, 0, st, wu, scale, wo, n8);
            }
            rc = check_launch(name);
        }
        if (rc == VOX_CUDA_OK) {
            GemmArgs a = q.g;
            a.f16 = 1;
            GemmPlan p;
            rc = gemm_plan(xh, cols, w16, cols, a, kEpiF32, p, name);
            if (rc == VOX_CUDA_OK) rc = gemm_run(p, st, name);
        }
        cudaFreeAsync(buf, st);
        return rc;
    }
    // Work split. T output tiles of 128 x 256 on P (the SM count) persistent CTAs leave the last wave T % P tiles wide
    // (512 x 12288: 192 tiles, 44 of 148 CTAs busy in the second wave; 512 x 4096: 64 tiles, one wave of 64). The T % P
    // tail tiles are cut instead into s = min(P / (T % P), K steps / 4, 8) K-ranges each, so every CTA takes its whole
    // tiles and at most one piece; the pieces' f32 partials are summed in a fixed order by gemm_q_fixup_kernel.
    // VOX_CUDA_GEMMQ_SPLIT=0 keeps whole tiles.
    {
        const int64_t mt = (m + kBM - 1) / kBM, nt = (rows + kQBN - 1) / kQBN, tiles = mt * nt, kt = (cols + kBK - 1) / kBK;
        const int64_t P = sm_count();
        const int64_t full = tiles / P * P, rem = tiles - full;
        int64_t s = rem ? P / rem : 1;
        if (s > kt / 4) s = kt / 4;
        if (s > 8) s = 8;
        const char *es = std::getenv("VOX_CUDA_GEMMQ_SPLIT");
        if (es && es[0] == '0') s = 1;
        VOX_REQUIRE(tiles < (int64_t(1) << 30), std::string(name) + ": shape too large");
        if (s >= 2) q.full = int(full), q.rem = int(rem), q.splits = int(s), q.items = int(full + rem * s);
        else q.full = int(tiles), q.rem = 1, q.splits = 1, q.items = int(tiles);
    }
    // x rounded to f16 once, and the pieces' partials, in stream-ordered scratch from the device's memory pool (freed,
    // stream-ordered, after the GEMM)
    void *xh = nullptr;
    const int64_t n4 = m * cols / 4;
    const size_t xh_bytes = (size_t(m * cols * 2) + 255) & ~size_t(255);
    const size_t part_bytes = q.splits > 1 ? size_t(q.rem) * q.splits * kBM * kQBN * sizeof(float) : 0;
    if (cudaMallocAsync(&xh, xh_bytes + part_bytes, st) != cudaSuccess) return check_launch(name);
    q.part = part_bytes ? reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(xh) + xh_bytes) : nullptr;
    launch_k(q_x_to_f16_kernel, grid_for(n4, 256, 4), 256, 0, st, reinterpret_cast<const float4 *>(x), reinterpret_cast<uint2 *>(xh), n4);
    int rc = check_launch(name);
    CUtensorMap tx, tw;
    if (rc == VOX_CUDA_OK) rc = bf16_map(xh, cols, m, 1, cols, kBM, tx, name, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    if (rc == VOX_CUDA_OK)
        rc = plain_map(w, CU_TENSOR_MAP_DATA_TYPE_UINT8, q4 ? cols / 2 : cols, rows, q4 ? cols / 2 : cols, q4 ? kBK / 2 : kBK, kQBN, tw, name);
    if (rc == VOX_CUDA_OK) {
        const bool f16 = scale_dtype == VOX_CUDA_F16;
        if (q4) rc = f16 ? launch_q<true, true>(tx, tw, q, st, name) : launch_q<true, false>(tx, tw, q, st, name);
        else rc = f16 ? launch_q<false, true>(tx, tw, q, st, name) : launch_q<false, false>(tx, tw, q, st, name);
    }
    cudaFreeAsync(xh, st);
    return rc;
}

int gemm_take_device_error(unsigned int *flags) { return take_device_error(flags); }

}  // namespace voxcuda

using namespace voxcuda;

extern "C" int vox_cuda_gemm_bf16(const void *x, const void *w, const float *bias, void *y, int64_t m, int64_t n, int64_t k, int act,
                                  int out_dtype, void *stream) {
    VOX_REQUIRE(m >= 0 && n > 0 && k > 0 && m < (int64_t(1) << 31) && n < (int64_t(1) << 31) && k < (int64_t(1) << 31),
                "vox_cuda_gemm_bf16: bad shape");
    VOX_REQUIRE(is_act_dtype(out_dtype), "vox_cuda_gemm_bf16: out_dtype must be F32 or BF16");
    VOX_REQUIRE(act >= VOX_CUDA_GEMM_NONE && act <= VOX_CUDA_GEMM_GELU_TANH, "vox_cuda_gemm_bf16: unknown activation");
    if (m == 0) return VOX_CUDA_OK;
    GemmArgs a;
    a.M = int(m), a.N = int(n), a.K = int(k);
    a.y = y, a.ldy = n, a.bias = bias;
    const bool f32 = out_dtype == VOX_CUDA_F32;
    const int epi = act == VOX_CUDA_GEMM_NONE ? (f32 ? kEpiF32 : kEpiBf16)
                    : act == VOX_CUDA_GEMM_GELU_ERF ? (f32 ? kEpiGeluErfF32 : kEpiGeluErf)
                                                    : (f32 ? kEpiGeluTanhF32 : kEpiGeluTanh);
    GemmPlan p;
    const int rc = gemm_plan(x, k, w, k, a, epi, p, "vox_cuda_gemm_bf16");
    if (rc != VOX_CUDA_OK) return rc;
    return gemm_run(p, reinterpret_cast<cudaStream_t>(stream), "vox_cuda_gemm_bf16");
}

extern "C" int vox_cuda_gemm_q8(const int8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y, int64_t rows,
                                int64_t cols, int64_t m, int accumulate, void *stream) {
    return gemm_q(false, w, scale, scale_dtype, bias, x, y, rows, cols, m, accumulate, reinterpret_cast<cudaStream_t>(stream), "vox_cuda_gemm_q8");
}

extern "C" int vox_cuda_gemm_q4(const uint8_t *w, const void *scale, int scale_dtype, const float *bias, const float *x, float *y, int64_t rows,
                                int64_t cols, int64_t m, int accumulate, void *stream) {
    return gemm_q(true, w, scale, scale_dtype, bias, x, y, rows, cols, m, accumulate, reinterpret_cast<cudaStream_t>(stream), "vox_cuda_gemm_q4");
}
