// GEMM on the 5th-generation tensor cores: y[z][M][N] = x[z][M][K] . W[g][N][K]^T (+ bias) with a fused epilogue,
// bf16 operands, f32 accumulation in tensor memory. It replaces the projections Vox records as GEMM dispatches in its
// GPU F5 step (gpu_f5.cpp:287-322, gemm(): shaders/gemmb.comp:1-99, with its bias and GELU flags) and the grouped
// position convolutions' GEMMs (shaders/convgemm.comp).
//
// One CTA per SM, persistent over output tiles of 128 rows x BN columns (BN 64, 128 or 256), tiles with the same W
// columns taken by neighbouring CTAs so a weight tile is read from HBM once and then from L2. Six warps:
//   warp 0      tensor copies (TMA): for every K step of 64, the x tile [128][64] and the W tile [BN][64], both in the
//               128-byte swizzle, into a ring of STAGES shared-memory stages (mbarrier full/empty pairs);
//   warp 1      one thread issues tcgen05.mma (M 128, N BN, K 16; four per K step) into one of two TMEM accumulators
//               and commits each stage back to the copy warp, and each finished tile to the epilogue;
//   warps 2..5  the epilogue: each thread reads its output row from TMEM (warp w reads lanes 32 (w % 4) ..), applies
//               bias / RoPE / GELU and stores it; the accumulator goes back to the MMA thread, which meanwhile has
//               started the next tile in the other accumulator.
// Every wait is bounded; a wait that gives up sets the device error flag and the CTA winds down (its copies and MMAs
// in flight are waited for, bounded, before its shared and tensor memory are released). No copy is broadcast across
// a cluster.
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
    static constexpr int STAGES = BN == 256 ? 4 : BN == 128 ? 6 : 8;
    static constexpr uint32_t B_BYTES = BN * kBK * 2;
    static constexpr uint32_t STAGE = kABytes + B_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
    static constexpr size_t SMEM = size_t(STAGES) * STAGE + 1024 + 256;
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

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

// The epilogue of 32 consecutive columns [c0, c0 + 32) of output row `row` (acc: f32 bit patterns).
template <int EPI>
__device__ __forceinline__ void epilogue32(const GemmArgs &g, const uint32_t (&acc)[32], int row, int c0, int zb, int zg) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(acc[i]);
    const int nv = min(32, g.N - c0);  // valid columns
    if (g.bias) {
        const float *b = g.bias + int64_t(zg) * g.N + c0;
        if (nv == 32 && (reinterpret_cast<uintptr_t>(b) & 15u) == 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 bb = __ldg(reinterpret_cast<const float4 *>(b) + q);
                v[4 * q] += bb.x, v[4 * q + 1] += bb.y, v[4 * q + 2] += bb.z, v[4 * q + 3] += bb.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (i < nv) v[i] += __ldg(b + i);
        }
    }
    if constexpr (EPI == kEpiQkvRope) {
        const int part = c0 / g.inner, ci = c0 - part * g.inner, head = ci / g.hd;
        if (part < 2 && head < g.rope_heads) {  // pairs (2j, 2j + 1) of the head, j = (ci % hd) / 2 ..
            const float2 *cs = g.cs + int64_t(row % g.frames) * (g.hd / 2) + (ci % g.hd) / 2;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float2 c = __ldg(cs + j);
                const float x0 = v[2 * j], x1 = v[2 * j + 1];
                v[2 * j] = __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(x1, c.y));  // f5.cpp:696-701, CPU rounding
                v[2 * j + 1] = __fadd_rn(__fmul_rn(x1, c.x), __fmul_rn(x0, c.y));
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
    const int64_t off = int64_t(zb) * g.y_bstride + int64_t(zg) * g.y_gstride + int64_t(row) * g.ldy + c0;
    if constexpr (EPI == kEpiF32 || EPI == kEpiGeluTanhF32 || EPI == kEpiGeluErfF32) {
        float *y = reinterpret_cast<float *>(g.y) + off;
        if (nv == 32 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                if (g.accumulate) {
                    const float4 p = reinterpret_cast<const float4 *>(y)[q];
                    o.x += p.x, o.y += p.y, o.z += p.z, o.w += p.w;
                }
                reinterpret_cast<float4 *>(y)[q] = o;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (i < nv) y[i] = g.accumulate ? y[i] + v[i] : v[i];
        }
    } else {
        uint16_t *y = reinterpret_cast<uint16_t *>(g.y) + off;
        if (nv == 32 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
                reinterpret_cast<uint4 *>(y)[q] = make_uint4(pack_bf16(v[8 * q], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                                                             pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7]));
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (i < nv) y[i] = to_bf16(v[i]);
        }
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                                                                  const GemmArgs g) {
    using C = Cfg<BN>;
    constexpr uint32_t kIdesc = umma_idesc_bf16(kBM, BN);
    extern __shared__ uint8_t gemm_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t s0 = smem_addr(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE);
    uint64_t *empty = full + C::STAGES;
    uint64_t *tfull = empty + C::STAGES;  // [2]: accumulator a holds a finished tile
    uint64_t *tempty = tfull + 2;         // [2]: accumulator a has been read out
    uint64_t *drain = tempty + 2;         // wind-down: every MMA issued has completed
    uint32_t *tslot = reinterpret_cast<uint32_t *>(drain + 1);
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
    pdl_enter();  // the previous grid (its outputs, and the tensor memory it held) is complete
    if (warp == 0) tmem_alloc(tslot, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    bool ok = true;

    if (warp == 0) {
        // ---- tensor copies
        uint32_t it = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            const Tile tl = tile_of(t, mt, nt, g.groups);
            for (int kc = 0; kc < kt; ++kc, ++it) {
                const int s = int(it % C::STAGES);
                const uint32_t u = it / C::STAGES;
                if (!mbar_wait_warp(&empty[s], (u & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t sa = s0 + uint32_t(s) * C::STAGE;
                    mbar_arrive_expect_tx(&full[s], C::STAGE);
                    tma_load_3d(sa, &ta, kc * kBK, tl.m0, tl.z, &full[s]);
                    tma_load_3d(sa + kABytes, &tb, kc * kBK, tl.ni * BN, tl.zg, &full[s]);
                }
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
                if (lane == 0) {
                    const uint32_t sa = s0 + uint32_t(s) * C::STAGE, sb = sa + kABytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        umma_bf16(dcol, umma_desc(sa + 32 * k, 16, 1024), umma_desc(sb + 32 * k, 16, 1024), kIdesc, (kc | k) != 0);
                    umma_commit(&empty[s]);  // the stage returns to the copy warp when these MMAs have read it
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) umma_commit(&tfull[a]);
            __syncwarp();
        }
        if (!ok) {  // wind-down: every MMA issued completes before the tensor memory is released
            if (lane == 0) umma_commit(drain);
            __syncwarp();
            mbar_wait_warp(drain, 0);
        }
    } else {
        // ---- epilogue: thread = output row 32 (warp % 4) + lane of the tile
        const int q = warp & 3;
        uint32_t tc = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
            const uint32_t a = tc & 1u, v = tc >> 1;
            if (!mbar_wait_warp(&tfull[a], v & 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const Tile tl = tile_of(t, mt, nt, g.groups);
            const int row = tl.m0 + 32 * q + lane;
            const uint32_t taddr = tmem + (uint32_t(32 * q) << 16) + a * BN;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                const int c0 = tl.ni * BN + c;
                if (c0 >= g.N) break;  // warp-uniform
                uint32_t r[32];
                tmem_ld32(taddr + uint32_t(c), r);
                tmem_wait_ld();
                if (row < g.M) epilogue32<EPI>(g, r, row, c0, tl.zb, tl.zg);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
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

// 3-D bf16 map of planes [depth][rows][cols] (row pitch ld elements, plane pitch rows * ld), box 64 x box_rows x 1,
// 128-byte swizzle, zero fill past every edge.
int bf16_map(const void *base, int64_t cols, int64_t rows, int64_t depth, int64_t ld, int box_rows, CUtensorMap &m, const char *name) {
    auto fn = encode();
    if (!fn) return set_error(VOX_CUDA_ERR_DEVICE, std::string(name) + ": cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(depth)};
    const cuuint64_t strides[2] = {cuuint64_t(ld) * 2, cuuint64_t(ld) * 2 * cuuint64_t(rows)};
    const cuuint32_t box[3] = {uint32_t(kBK), uint32_t(box_rows), 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VOX_CUDA_ERR_ARG, std::string(name) + ": tensor map rejected (code " + std::to_string(int(r)) + ")");
    return VOX_CUDA_OK;
}

template <int BN, int EPI>
int launch(const GemmPlan &p, cudaStream_t st, const char *name) {
    auto kern = gemm_tc_kernel<BN, EPI>;
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
    launch_k(kern, grid, kGemmThreads, Cfg<BN>::SMEM, st, p.ta, p.tb, p.a);
    return check_launch(name);
}

template <int EPI>
int launch_bn(const GemmPlan &p, cudaStream_t st, const char *name) {
    if (p.bn == 64) return launch<64, EPI>(p, st, name);
    if (p.bn == 256) return launch<256, EPI>(p, st, name);
    return launch<128, EPI>(p, st, name);
}

}  // namespace

int gemm_plan(const void *x, int64_t ldx, const void *w, int64_t ldw, const GemmArgs &a, int epi, GemmPlan &plan, const char *name) {
    VOX_REQUIRE(a.M > 0 && a.N > 0 && a.K > 0 && a.batches > 0 && a.groups > 0, std::string(name) + ": bad GEMM shape");
    VOX_REQUIRE(x && w && a.y, std::string(name) + ": NULL pointer");
    VOX_REQUIRE(a.K % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 && ldx >= a.K && ldw >= a.K && aligned16(x) && aligned16(w),
                std::string(name) + ": x and W need 16-byte aligned rows (K and the row pitches multiples of 8)");
    VOX_REQUIRE(epi >= kEpiF32 && epi <= kEpiGeluErfF32, std::string(name) + ": unknown epilogue");
    if (epi == kEpiQkvRope)
        VOX_REQUIRE(a.cs && a.inner > 0 && a.inner % 32 == 0 && a.hd % 32 == 0 && a.N == 3 * a.inner && a.frames > 0,
                    std::string(name) + ": RoPE epilogue needs 3 inner columns with inner and hd multiples of 32");
    plan.a = a;
    plan.epi = epi;
    // tile width: fewest tile columns per SM-wave (ceil(tiles / SMs) * BN), the wider tile on a tie
    const int64_t sms = sm_count(), mt = (a.M + kBM - 1) / kBM, z = int64_t(a.batches) * a.groups;
    int best = 256;
    int64_t best_cost = -1;
    for (int bn : {256, 128, 64}) {
        if (bn > 64 && a.N <= bn / 2) continue;  // mostly empty tiles
        const int64_t tiles = mt * ((a.N + bn - 1) / bn) * z;
        const int64_t cost = (tiles + sms - 1) / sms * bn;
        if (best_cost < 0 || cost < best_cost) best = bn, best_cost = cost;
    }
    // VOX_CUDA_GEMM_BN = 64 / 128 / 256 forces the tile width (for comparisons)
    static const int forced = [] {
        const char *e = std::getenv("VOX_CUDA_GEMM_BN");
        const int v = e ? std::atoi(e) : 0;
        return v == 64 || v == 128 || v == 256 ? v : 0;
    }();
    plan.bn = forced ? forced : best;
    int rc = bf16_map(x, a.K, a.M, z, ldx, kBM, plan.ta, name);
    if (rc != VOX_CUDA_OK) return rc;
    return bf16_map(w, a.K, a.N, a.groups, ldw, plan.bn, plan.tb, name);
}

int gemm_run(const GemmPlan &p, cudaStream_t st, const char *name) {
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
