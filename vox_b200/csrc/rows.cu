// The row operators on the TMA row pipeline (tma.cuh): RMSNorm, LayerNorm (affine / modulate), the fused adaLN
// block, and the scaled causal softmax. One warp per row; the row (and the adaLN residual row) arrives in shared
// memory by bulk copy STAGES rows ahead, is moved into registers (VPL 16-byte vectors per lane), reduced with
// warp shuffles, and written with 16-byte streaming stores.
//
// Arithmetic follows the code it replaces: RMSNorm sums x^2 in f32 (kernels.cpp:707-712); LayerNorm and adaLN take
// the two-pass mean and variance (kernels.cpp:714-723, nn.cpp:252-258, f5.cpp:622-628) in f32 with warp
// butterflies, as Vox's own GPU shaders do (f5ln.comp, layernorm.comp) — the CPU accumulates in f64, which moves the
// statistics by ~1e-7 relative; the softmax takes max, exp(x - max), f32 sum and multiplies by 1/sum
// (kernels.cpp:725-732) over the visible prefix only (kernels.cpp:812-819), with exp evaluated as
// 2^((x - max) log2 e) on the SFU (relative error ~3e-7 against expf). Arithmetic runs two elements per instruction
// (packed f32x2: FADD2 / FMUL2 / FFMA2). RMSNorm's output w * (x * inv) and the softmax's outputs round as the CPU
// does (their sums of squares and of exponentials may be fused into FMAs); the LayerNorm / adaLN epilogues use fused
// multiply-adds ((x - mean)/sigma as fma(x, 1/sigma, -mean/sigma), then one FMA
// per affine step) and 1/sigma = rsqrt(var + eps): differences from the CPU of about one f32 ulp, far inside the
// 1e-5 (f32) and 1e-2 (bf16) tolerances, for about half the instructions.
#include <math.h>

#include <cstdlib>

#include "gemm.cuh"
#include "rows.cuh"
#include "tma.cuh"
#include "sfu.cuh"

namespace voxcuda {
namespace {

constexpr int kStages = 2;

template <int DT, int VPL, int KIND>
struct NormOp {
    // gated bf16 adaLN (x and residual staged, 4 KB a stage): registers capped for 5 CTAs per SM (96 a thread, no
    // spill), which keeps 20 warps per SM in flight on this latency-bound row
    static constexpr int kMinBlocks = (KIND == kAdaLnGated && DT == VOX_CUDA_BF16 && VPL <= 4) ? 5 : 1;
    NormArgs a;
    uint32_t row_bytes;  // n * element size (multiple of 16)

    __device__ __forceinline__ void issue(int64_t r, uint8_t *buf, uint64_t *bar) const {
        const char *xr = reinterpret_cast<const char *>(a.x) + r * int64_t(row_bytes);
        if (KIND == kAdaLnGated) {
            mbar_arrive_expect_tx(bar, 2 * row_bytes);
            bulk_g2s(buf, xr, row_bytes, bar);
            bulk_g2s(buf + row_bytes, reinterpret_cast<const char *>(a.res) + r * int64_t(row_bytes), row_bytes, bar);
        } else {
            mbar_arrive_expect_tx(bar, row_bytes);
            bulk_g2s(buf, xr, row_bytes, bar);
        }
    }

    template <class Next>
    __device__ __forceinline__ void run(int64_t r, const uint8_t *buf, int lane, Next next) const {
        constexpr int W = Vec<DT>::N, PW = W / 2;  // values and float pairs per 16-byte vector
        constexpr int ES = DT == VOX_CUDA_F32 ? 4 : 2;
        const int nvec = int(a.n / W);
        float2 xv[VPL][PW];
        uint4 rres[VPL];  // the residual stays packed until the epilogue
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int j = lane + 32 * k;
            const uint4 raw = j < nvec ? *reinterpret_cast<const uint4 *>(buf + j * 16) : make_uint4(0, 0, 0, 0);
            unpack2<DT>(raw, xv[k]);
            if (KIND == kAdaLnGated) rres[k] = j < nvec ? *reinterpret_cast<const uint4 *>(buf + row_bytes + j * 16) : make_uint4(0, 0, 0, 0);
        }
        next();
        float2 negmean = bc2(0.f), inv2;
        if (KIND == kRms) {
            float2 ss = bc2(0.f);
#pragma unroll
            for (int k = 0; k < VPL; ++k)
#pragma unroll
                for (int p = 0; p < PW; ++p) ss = add2(ss, mul2(xv[k][p], xv[k][p]));
            const float sum = warp_sum(__fadd_rn(ss.x, ss.y));
            inv2 = bc2(__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, float(a.n)), a.eps))));
        } else {
            // two-pass mean / variance on the row in registers, f32 butterflies (as f5ln.comp / layernorm.comp)
            float2 sm = bc2(0.f);
#pragma unroll
            for (int k = 0; k < VPL; ++k)
#pragma unroll
                for (int p = 0; p < PW; ++p) sm = add2(sm, xv[k][p]);
            const float meanf = warp_sum(__fadd_rn(sm.x, sm.y)) * a.inv_n;
            negmean = bc2(-meanf);
            float2 v = bc2(0.f);
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                if (lane + 32 * k < nvec) {
#pragma unroll
                    for (int p = 0; p < PW; ++p) {
                        const float2 d = add2(xv[k][p], negmean);
                        v = fma2(d, d, v);
                    }
                }
            }
            const float var = warp_sum(__fadd_rn(v.x, v.y)) * a.inv_n;
            inv2 = bc2(rsqrtf(var + a.eps));
        }
        const float2 one = bc2(1.0f);
        const float2 nmi = mul2(negmean, inv2);  // -mean / sigma: (x - mean) / sigma = fma(x, inv, -mean * inv)
        const int64_t batch = (KIND >= kAdaLn) ? int64_t(a.tdiv.div(uint32_t(r))) : 0;  // rows < 2^32 (launcher)
        char *yr = reinterpret_cast<char *>(a.y) + r * int64_t(row_bytes);
        // adaLN parameter vectors of the batch: loaded one k-step ahead of their use (ordered loads, served by L1)
        const char *scp = reinterpret_cast<const char *>(a.scale) + batch * a.n * ES;
        const char *shp = reinterpret_cast<const char *>(a.shift) + batch * a.n * ES;
        const char *gp = reinterpret_cast<const char *>(a.gate) + batch * a.n * ES;
        uint4 psc, psh, pg;
        if (KIND >= kAdaLn && lane < nvec) {
            psc = ld_param_ordered(scp + lane * 16);
            psh = ld_param_ordered(shp + lane * 16);
            if (KIND == kAdaLnGated) pg = ld_param_ordered(gp + lane * 16);
        }
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int j = lane + 32 * k;
            if (j < nvec) {
                float2 o[PW];
                if (KIND <= kLnMod) {
                    // f32 weight / bias vectors (Vox keeps them as const float *): PW pairs from ordered L1 loads
                    float2 wv[PW], bv[PW];
#pragma unroll
                    for (int q = 0; q < PW; q += 2) {
                        const uint4 wq = a.w ? ld_param_ordered(a.w + j * W + 2 * q) : as_u4(make_float4(1.f, 1.f, 1.f, 1.f));
                        const uint4 bq = a.b ? ld_param_ordered(a.b + j * W + 2 * q) : make_uint4(0, 0, 0, 0);
                        unpack2<VOX_CUDA_F32>(wq, wv + q);
                        unpack2<VOX_CUDA_F32>(bq, bv + q);
                    }
#pragma unroll
                    for (int p = 0; p < PW; ++p) {
                        if (KIND == kRms) {
                            o[p] = mul2(wv[p], mul2(xv[k][p], inv2));                   // kernels.cpp:711, CPU rounding
                        } else {
                            const float2 nrm = fma2(xv[k][p], inv2, nmi);
                            if (KIND == kLnMod) o[p] = fma2(add2(one, wv[p]), nrm, bv[p]);  // nn.cpp:262
                            else if (a.w) o[p] = fma2(nrm, wv[p], bv[p]);               // kernels.cpp:722
                            else o[p] = a.b ? add2(nrm, bv[p]) : nrm;                   // no weight: nn.cpp:262
                        }
                    }
                } else {
                    float2 sc[PW], sh[PW], gv[PW], rv[PW];
                    unpack2<DT>(psc, sc);
                    unpack2<DT>(psh, sh);
                    if (KIND == kAdaLnGated) {
                        unpack2<DT>(pg, gv);
                        unpack2<DT>(rres[k], rv);
                    }
                    const int jn = j + 32;
                    if (k + 1 < VPL && jn < nvec) {  // next k-step's parameters, in flight during this step's math
                        psc = ld_param_ordered(scp + jn * 16);
                        psh = ld_param_ordered(shp + jn * 16);
                        if (KIND == kAdaLnGated) pg = ld_param_ordered(gp + jn * 16);
                    }
#pragma unroll
                    for (int p = 0; p < PW; ++p) {
                        const float2 nrm = fma2(xv[k][p], inv2, nmi);
                        const float2 m = fma2(nrm, add2(one, sc[p]), sh[p]);          // f5.cpp:630
                        o[p] = KIND == kAdaLnGated ? fma2(gv[p], m, rv[p]) : m;       // f5.cpp:674
                    }
                }
                st_stream(yr + j * 16, pack2<DT>(o));
            }
        }
    }
};

// Gated adaLN with the batch's parameters folded once per CTA. y = res + g * ((x - mean) / sigma * (1 + s) + h)
// = res + A * n + C with A = g * (1 + s), C = g * h (f5.cpp:630, 674 regrouped; n = (x - mean) / sigma). A CTA takes a
// contiguous range of rows, so all its rows but those past a batch boundary share one batch: it computes that batch's
// A and C once into shared memory (f32), and each row's epilogue is one FMA and one add per element instead of
// unpacking three parameter vectors. Rows of a second batch in the range take NormOp's epilogue (parameters from
// global memory). Staging, waits and statistics are those of the row pipeline.
template <int DT, int VPL>
__global__ void __launch_bounds__(kPipeWarps * 32, VPL <= 4 ? 5 : 3) adaln_ac_kernel(NormArgs a, uint32_t row_bytes) {
    constexpr int STAGES = kStages;
    constexpr int W = Vec<DT>::N, PW = W / 2;
    constexpr int ES = DT == VOX_CUDA_F32 ? 4 : 2;
    pdl_enter();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t stage_bytes = 2 * row_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * STAGES;
    uint8_t *bufs = smem + pipe_bar_bytes(STAGES) + size_t(warp) * STAGES * stage_bytes;
    float *ac = reinterpret_cast<float *>(smem + pipe_bar_bytes(STAGES) + size_t(kPipeWarps) * STAGES * stage_bytes);  // A[n], C[n]
    const int64_t r0 = a.rows * int64_t(blockIdx.x) / gridDim.x, r1 = a.rows * int64_t(blockIdx.x + 1) / gridDim.x;
    const int nvec = int(a.n / W);
    auto issue = [&](int64_t r, uint8_t *buf, uint64_t *bar) {
        mbar_arrive_expect_tx(bar, 2 * row_bytes);
        bulk_g2s(buf, reinterpret_cast<const char *>(a.x) + r * int64_t(row_bytes), row_bytes, bar);
        bulk_g2s(buf + row_bytes, reinterpret_cast<const char *>(a.res) + r * int64_t(row_bytes), row_bytes, bar);
    };
    // this warp's rows: r0 + warp, r0 + warp + kPipeWarps, ...
    const int64_t first = r0 + warp;
    const int64_t stall = lane == 0 ? g_stall_row : -1;  // test hook (-1 in normal use)
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        mbar_init_fence();
#pragma unroll
        for (int s = 0; s < STAGES; ++s) {
            if (first + s * kPipeWarps == stall) mbar_expect_tx(&bars[s], 16);
            if (first + s * kPipeWarps < r1) issue(first + s * kPipeWarps, bufs + s * stage_bytes, &bars[s]);
        }
    }
    uint32_t pending = 0;
#pragma unroll
    for (int t = 0; t < STAGES; ++t)
        if (first + t * kPipeWarps < r1) pending |= 1u << t;
    // A and C of the range's first batch, while the first rows are in flight. Pairs 2q, 2q + 1 of 16-byte vector v sit
    // in float4 q * nvec + v, so one epilogue read of the 32 lanes (vectors lane + 32 k) is 512 contiguous bytes: four
    // shared-memory wavefronts, the minimum for 16 bytes a lane (a vector-major table, lanes 32 bytes apart, took
    // eight wavefronts for every 8 bytes a lane).
    const int64_t batch0 = r0 < r1 ? int64_t(a.tdiv.div(uint32_t(r0))) : 0;
    if (r0 < r1) {
        const char *scp = reinterpret_cast<const char *>(a.scale) + batch0 * a.n * ES;
        const char *shp = reinterpret_cast<const char *>(a.shift) + batch0 * a.n * ES;
        const char *gp = reinterpret_cast<const char *>(a.gate) + batch0 * a.n * ES;
        for (int v = threadIdx.x; v < nvec; v += kPipeWarps * 32) {
            float2 sc[PW], sh[PW], gv[PW];
            unpack2<DT>(ld_param(scp + v * 16), sc);
            unpack2<DT>(ld_param(shp + v * 16), sh);
            unpack2<DT>(ld_param(gp + v * 16), gv);
#pragma unroll
            for (int q = 0; q < PW / 2; ++q) {
                const float2 a0 = mul2(gv[2 * q], add2(bc2(1.0f), sc[2 * q])), a1 = mul2(gv[2 * q + 1], add2(bc2(1.0f), sc[2 * q + 1]));
                const float2 c0 = mul2(gv[2 * q], sh[2 * q]), c1 = mul2(gv[2 * q + 1], sh[2 * q + 1]);
                reinterpret_cast<float4 *>(ac)[q * nvec + v] = make_float4(a0.x, a0.y, a1.x, a1.y);
                reinterpret_cast<float4 *>(ac + a.n)[q * nvec + v] = make_float4(c0.x, c0.y, c1.x, c1.y);
            }
        }
    }
    __syncthreads();
    uint32_t parity = 0;
    int s = 0;
    for (int64_t r = first; r < r1; r += kPipeWarps) {
        if (!mbar_wait_warp(&bars[s], (parity >> s) & 1u)) {
            // give up: every copy of the warp still in flight lands (bounded), the one waited for included
            for (int t = 0; t < STAGES; ++t)
                if ((pending >> t) & 1u) mbar_wait_warp(&bars[t], (parity >> t) & 1u);
            return;
        }
        parity ^= 1u << s;
        pending &= ~(1u << s);
        uint8_t *buf = bufs + s * stage_bytes;
        float2 xv[VPL][PW];
        uint4 rres[VPL];
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int j = lane + 32 * k;
            const uint4 raw = j < nvec ? *reinterpret_cast<const uint4 *>(buf + j * 16) : make_uint4(0, 0, 0, 0);
            unpack2<DT>(raw, xv[k]);
            rres[k] = j < nvec ? *reinterpret_cast<const uint4 *>(buf + row_bytes + j * 16) : make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
        const int64_t r_next = r + int64_t(STAGES) * kPipeWarps;
        if (r_next < r1) {
            if (lane == 0) {
                fence_proxy_async();
                if (r_next == stall) mbar_expect_tx(&bars[s], 16);
                issue(r_next, buf, &bars[s]);
            }
            pending |= 1u << s;
        }
        // two-pass mean / variance in f32 on the row in registers (as NormOp)
        float2 sm = bc2(0.f);
#pragma unroll
        for (int k = 0; k < VPL; ++k)
#pragma unroll
            for (int p = 0; p < PW; ++p) sm = add2(sm, xv[k][p]);
        const float meanf = warp_sum(__fadd_rn(sm.x, sm.y)) * a.inv_n;
        const float2 negmean = bc2(-meanf);
        float2 vv = bc2(0.f);
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if (lane + 32 * k < nvec) {
#pragma unroll
                for (int p = 0; p < PW; ++p) {
                    const float2 d = add2(xv[k][p], negmean);
                    vv = fma2(d, d, vv);
                }
            }
        }
        const float var = warp_sum(__fadd_rn(vv.x, vv.y)) * a.inv_n;
        const float2 inv2 = bc2(rsqrtf(var + a.eps));
        const float2 nmi = mul2(negmean, inv2);
        const int64_t batch = int64_t(a.tdiv.div(uint32_t(r)));
        char *yr = reinterpret_cast<char *>(a.y) + r * int64_t(row_bytes);
        if (batch == batch0) {
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const int j = lane + 32 * k;
                if (j < nvec) {
                    float2 rv[PW], o[PW];
                    unpack2<DT>(rres[k], rv);
                    const float4 *A = reinterpret_cast<const float4 *>(ac) + j;
                    const float4 *Cc = reinterpret_cast<const float4 *>(ac + a.n) + j;
#pragma unroll
                    for (int q = 0; q < PW / 2; ++q) {
                        const float4 av = A[q * nvec], cv = Cc[q * nvec];
                        o[2 * q] = add2(fma2(make_float2(av.x, av.y), fma2(xv[k][2 * q], inv2, nmi), make_float2(cv.x, cv.y)), rv[2 * q]);
                        o[2 * q + 1] = add2(fma2(make_float2(av.z, av.w), fma2(xv[k][2 * q + 1], inv2, nmi), make_float2(cv.z, cv.w)), rv[2 * q + 1]);
                    }
                    st_stream(yr + j * 16, pack2<DT>(o));
                }
            }
        } else {  // a row past the range's batch boundary: the parameters from global memory
            const char *scp = reinterpret_cast<const char *>(a.scale) + batch * a.n * ES;
            const char *shp = reinterpret_cast<const char *>(a.shift) + batch * a.n * ES;
            const char *gp = reinterpret_cast<const char *>(a.gate) + batch * a.n * ES;
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const int j = lane + 32 * k;
                if (j < nvec) {
                    float2 sc[PW], sh[PW], gv[PW], rv[PW], o[PW];
                    unpack2<DT>(ld_param(scp + j * 16), sc);
                    unpack2<DT>(ld_param(shp + j * 16), sh);
                    unpack2<DT>(ld_param(gp + j * 16), gv);
                    unpack2<DT>(rres[k], rv);
#pragma unroll
                    for (int p = 0; p < PW; ++p) {
                        const float2 A = mul2(gv[p], add2(bc2(1.0f), sc[p])), Cc = mul2(gv[p], sh[p]);
                        o[p] = add2(fma2(A, fma2(xv[k][p], inv2, nmi), Cc), rv[p]);
                    }
                    st_stream(yr + j * 16, pack2<DT>(o));
                }
            }
        }
        s = (s + 1 == STAGES) ? 0 : s + 1;
    }
}

// VOX_CUDA_ADALN_AC=0 keeps the gated adaLN on NormOp's epilogue (for comparisons).
bool adaln_ac_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("VOX_CUDA_ADALN_AC");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <int DT, int VPL>
int launch_adaln_ac(const NormArgs &a, cudaStream_t st, const char *name) {
    const uint32_t row_bytes = uint32_t(a.n * (DT == VOX_CUDA_F32 ? 4 : 2));
    const size_t smem = pipe_bar_bytes(kStages) + size_t(kPipeWarps) * kStages * 2 * row_bytes + size_t(a.n) * 8;
    if (int64_t(smem) > smem_optin()) return kPipeNotApplicable;
    auto kern = adaln_ac_kernel<DT, VPL>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
        return check_launch(name);
    // one wave of CTAs, each a contiguous range of at least kPipeWarps rows
    const int64_t resident = resident_blocks((const void *)kern, kPipeWarps * 32, smem);
    const int64_t want = (a.rows + kPipeWarps - 1) / kPipeWarps;
    const int g = int(want < resident ? want : resident);
    launch_k(kern, g < 1 ? 1 : g, kPipeWarps * 32, smem, st, a, row_bytes);
    return check_launch(name);
}

// Visible keys of row r: min(n, r % q_len + pos0 + 1); rows < 2^32 (launcher), q_len's division precomputed.
__device__ __forceinline__ int64_t visible_len(int64_t r, int64_t n, int64_t q_len, const FastDiv &qdiv, int64_t pos0) {
    if (q_len <= 0) return n;
    const int64_t v = int64_t(qdiv.mod(uint32_t(r))) + pos0 + 1;
    return v < n ? v : n;
}

// FOLD (scale positive and finite): s x - max(s x) = s (x - max x), so the maximum is taken on the raw scores and the scale, log2 e
// and the maximum fold into one multiply-add per pair ahead of the SFU's 2^y: fma(x, s log2e, -max(x) s log2e). The
// argument differs from the CPU's (s x - max) log2 e by a rounding or two (relative change of the result ~1e-6 at the
// scores' range), inside the f32 tolerance. Other scales take the multiply, subtract and scale steps.
template <int VPL, bool FOLD = false>
struct SoftmaxOp {
    static constexpr int kMinBlocks = 1;
    const float *x;
    float *y;
    int64_t n, q_len, pos0;
    float scale;
    FastDiv qdiv;

    __device__ __forceinline__ void issue(int64_t r, uint8_t *buf, uint64_t *bar) const {
        const uint32_t bytes = uint32_t((visible_len(r, n, q_len, qdiv, pos0) * 4 + 15) / 16 * 16);  // only the visible prefix
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(buf, x + r * n, bytes, bar);
    }

    template <class Next>
    __device__ __forceinline__ void run(int64_t r, const uint8_t *buf, int lane, Next next) const {
        const int vis = int(visible_len(r, n, q_len, qdiv, pos0));
        const int vvec = (vis + 3) / 4;  // vectors holding a visible element
        const int nvec = int(n / 4);
        float2 v[VPL][2];
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int j = lane + 32 * k;
            const uint4 t = j < vvec ? *reinterpret_cast<const uint4 *>(buf + j * 16) : make_uint4(0, 0, 0, 0);
            unpack2<VOX_CUDA_F32>(t, v[k]);
        }
        next();
        // scaled scores (kernels.cpp:812-816), -inf past the visible prefix; vectors past it are skipped warp-uniformly
        const float2 s2 = bc2(scale);
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if (128 * (k + 1) <= vis) {  // the whole block of 32 vectors is visible: no mask
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    if (!FOLD) v[k][p] = mul2(s2, v[k][p]);
                    mx = fmaxf(mx, fmaxf(v[k][p].x, v[k][p].y));
                }
            } else if (32 * k < vvec) {  // the block holding the end of the visible prefix
                const int base = (lane + 32 * k) * 4;
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    float2 t = FOLD ? v[k][p] : mul2(s2, v[k][p]);
                    t.x = base + 2 * p < vis ? t.x : -INFINITY;
                    t.y = base + 2 * p + 1 < vis ? t.y : -INFINITY;
                    v[k][p] = t;
                    mx = fmaxf(mx, fmaxf(t.x, t.y));
                }
            }
        }
        mx = warp_max(mx);
        // exp(x - max) as 2^((x - max) * log2 e) on the SFU (exp of -inf is 0); float sum (kernels.cpp:728-729)
        constexpr float kLog2e = 1.4426950408889634f;
        const float sl = FOLD ? scale * kLog2e : kLog2e;
        const float2 nm = bc2(-mx), l2e = bc2(kLog2e), sl2 = bc2(sl), off = bc2(-(mx * sl));
        float2 sum2 = bc2(0.f);
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            if (32 * k < vvec) {
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    const float2 d = FOLD ? fma2(v[k][p], sl2, off) : mul2(add2(v[k][p], nm), l2e);
                    v[k][p] = make_float2(ex2_approx(d.x), ex2_approx(d.y));
                    sum2 = add2(sum2, v[k][p]);
                }
            }
        }
        const float sum = warp_sum(__fadd_rn(sum2.x, sum2.y));
        const float2 inv = bc2(__fdiv_rn(1.0f, sum));
        float *yr = y + r * n;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int j = lane + 32 * k;
            if (j < nvec) {
                float2 o[2] = {bc2(0.f), bc2(0.f)};
                if (32 * k < vvec) {
                    o[0] = mul2(v[k][0], inv);
                    o[1] = mul2(v[k][1], inv);
                }
                st_stream(yr + j * 4, pack2<VOX_CUDA_F32>(o));
            }
        }
    }
};

// Residual update + RMSNorm (kernels.cpp:822-825 then :833): the h row and the d row arrive together in one stage;
// h + d * ls rounds the product and the sum separately (scalar, so that no multiply-add is formed), as the CPU.
template <int DT, int VPL>
struct AddRmsOp {
    static constexpr int kMinBlocks = 1;
    AddRmsArgs a;
    uint32_t row_bytes;

    __device__ __forceinline__ void issue(int64_t r, uint8_t *buf, uint64_t *bar) const {
        mbar_arrive_expect_tx(bar, 2 * row_bytes);
        bulk_g2s(buf, reinterpret_cast<const char *>(a.h) + r * int64_t(row_bytes), row_bytes, bar);
        bulk_g2s(buf + row_bytes, reinterpret_cast<const char *>(a.d) + r * int64_t(row_bytes), row_bytes, bar);
    }

    template <class Next>
    __device__ __forceinline__ void run(int64_t r, const uint8_t *buf, int lane, Next next) const {
        constexpr int W = Vec<DT>::N, PW = W / 2;
        const int nvec = int(a.n / W);
        float2 hv[VPL][PW];
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int j = lane + 32 * k;
            float2 dv[PW];
            const uint4 rh = j < nvec ? *reinterpret_cast<const uint4 *>(buf + j * 16) : make_uint4(0, 0, 0, 0);
            const uint4 rd = j < nvec ? *reinterpret_cast<const uint4 *>(buf + row_bytes + j * 16) : make_uint4(0, 0, 0, 0);
            unpack2<DT>(rh, hv[k]);
            unpack2<DT>(rd, dv);
            if (a.ls) {
                float2 lv[PW];
#pragma unroll
                for (int q = 0; q < PW; q += 2)
                    unpack2<VOX_CUDA_F32>(j < nvec ? ld_param_ordered(a.ls + j * W + 2 * q) : make_uint4(0, 0, 0, 0), lv + q);
#pragma unroll
                for (int p = 0; p < PW; ++p)
                    hv[k][p] = make_float2(__fadd_rn(hv[k][p].x, __fmul_rn(dv[p].x, lv[p].x)),
                                           __fadd_rn(hv[k][p].y, __fmul_rn(dv[p].y, lv[p].y)));
            } else {
#pragma unroll
                for (int p = 0; p < PW; ++p) hv[k][p] = add2(hv[k][p], dv[p]);
            }
        }
        next();
        float2 ss = bc2(0.f);
#pragma unroll
        for (int k = 0; k < VPL; ++k)
#pragma unroll
            for (int p = 0; p < PW; ++p) ss = fma2(hv[k][p], hv[k][p], ss);
        const float sum = warp_sum(__fadd_rn(ss.x, ss.y));
        const float2 inv2 = bc2(__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, float(a.n)), a.eps))));
        char *hr = reinterpret_cast<char *>(a.h) + r * int64_t(row_bytes);
        char *xr = reinterpret_cast<char *>(a.xn) + r * int64_t(row_bytes);
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int j = lane + 32 * k;
            if (j < nvec) {
                float2 wv[PW], o[PW];
#pragma unroll
                for (int q = 0; q < PW; q += 2) unpack2<VOX_CUDA_F32>(ld_param_ordered(a.w + j * W + 2 * q), wv + q);
#pragma unroll
                for (int p = 0; p < PW; ++p) o[p] = mul2(wv[p], mul2(hv[k][p], inv2));  // kernels.cpp:711
                st_stream(hr + j * 16, pack2<DT>(hv[k]));
                st_stream(xr + j * 16, pack2<DT>(o));
            }
        }
    }
};

// Row sum / max / L2 norm in the fixed order of vox_cuda_row_reduce: lane l takes vectors l, l+32, ... in order,
// element k of a vector into accumulator k % 4, lane value (a0 + a1) + (a2 + a3), xor butterfly over the lanes.
// Reads the staged row from shared memory vector by vector (the row need not fit in registers).
template <int DT, int OP>
struct ReduceOp {
    static constexpr int kMinBlocks = 1;
    const void *x;
    float *out;
    int64_t n;
    uint32_t row_bytes;

    __device__ __forceinline__ void issue(int64_t r, uint8_t *buf, uint64_t *bar) const {
        mbar_arrive_expect_tx(bar, row_bytes);
        bulk_g2s(buf, reinterpret_cast<const char *>(x) + r * int64_t(row_bytes), row_bytes, bar);
    }

    __device__ __forceinline__ static float step(float acc, float v) {
        if (OP == VOX_CUDA_REDUCE_MAX) return fmaxf(acc, v);
        if (OP == VOX_CUDA_REDUCE_L2) return __fadd_rn(acc, __fmul_rn(v, v));
        return __fadd_rn(acc, v);
    }
    __device__ __forceinline__ static float join(float a, float b) { return OP == VOX_CUDA_REDUCE_MAX ? fmaxf(a, b) : __fadd_rn(a, b); }

    template <class Next>
    __device__ __forceinline__ void run(int64_t r, const uint8_t *buf, int lane, Next next) const {
        constexpr int W = Vec<DT>::N;
        const int nvec = int(n / W);
        const float init = OP == VOX_CUDA_REDUCE_MAX ? -INFINITY : 0.f;
        float acc[4] = {init, init, init, init};
#pragma unroll 4
        for (int j = lane; j < nvec; j += 32) {
            float f[W];
            Vec<DT>::unpack(*reinterpret_cast<const uint4 *>(buf + j * 16), f);
#pragma unroll
            for (int k = 0; k < W; ++k) acc[k % 4] = step(acc[k % 4], f[k]);
        }
        next();
        float v = join(join(acc[0], acc[1]), join(acc[2], acc[3]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = join(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) out[r] = OP == VOX_CUDA_REDUCE_L2 ? __fsqrt_rn(v) : v;
    }
};

template <int DT, int OP>
int reduce_pipe(const void *x, float *out, int64_t rows, int64_t n, cudaStream_t st) {
    const uint32_t row_bytes = uint32_t(n * (DT == VOX_CUDA_F32 ? 4 : 2));
    return launch_row_pipe<ReduceOp<DT, OP>, kStages>(ReduceOp<DT, OP>{x, out, n, row_bytes}, rows, row_bytes, st,
                                                       "vox_cuda_row_reduce");
}

// ------------------------------------------------------------------ few rows: one CTA per row

// For fewer rows than a resident wave has warps (BASELINE cfg1: 512 rows of 1024 on 148 SMs), a warp per row leaves
// the SMs nearly empty and every row's latency serial. Here a CTA takes one row and each thread VPT of its 16-byte
// vectors, so all loads of the launch are in flight at once; the statistics are folded by warp butterflies and then
// across the CTA's warps in warp order through shared memory (a fixed order), with the arithmetic of NormOp.
constexpr int kCtaRowMaxThreads = 1024;

template <int DT>
__device__ __forceinline__ float cta_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.f;
    t = warp_sum(t);
    __syncthreads();  // red is reused by the next fold
    return t;
}

template <int DT, int KIND, int VPT>
__global__ void __launch_bounds__(kCtaRowMaxThreads) norm_cta_kernel(NormArgs a, uint32_t row_bytes) {
    pdl_enter();
    constexpr int W = Vec<DT>::N, PW = W / 2;
    constexpr int ES = DT == VOX_CUDA_F32 ? 4 : 2;
    __shared__ float red[32];
    const int64_t r = blockIdx.x;
    const int nvec = int(a.n / W), t = threadIdx.x, nt = blockDim.x;
    const char *xr = reinterpret_cast<const char *>(a.x) + r * int64_t(row_bytes);
    const char *rr = reinterpret_cast<const char *>(a.res) + r * int64_t(row_bytes);
    float2 xv[VPT][PW];
    uint4 rres[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int j = t + nt * k;
        // coherent loads: y (and the adaLN residual) may alias x; each thread writes only the vectors it read
        unpack2<DT>(j < nvec ? ld_cg(xr + j * 16) : make_uint4(0, 0, 0, 0), xv[k]);
        if (KIND == kAdaLnGated) rres[k] = j < nvec ? ld_cg(rr + j * 16) : make_uint4(0, 0, 0, 0);
    }
    float2 negmean = bc2(0.f), inv2;
    if (KIND == kRms) {
        float2 ss = bc2(0.f);
#pragma unroll
        for (int k = 0; k < VPT; ++k)
#pragma unroll
            for (int p = 0; p < PW; ++p) ss = add2(ss, mul2(xv[k][p], xv[k][p]));
        const float sum = cta_sum<DT>(__fadd_rn(ss.x, ss.y), red);
        inv2 = bc2(__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, float(a.n)), a.eps))));
    } else {
        float2 sm = bc2(0.f);
#pragma unroll
        for (int k = 0; k < VPT; ++k)
#pragma unroll
            for (int p = 0; p < PW; ++p) sm = add2(sm, xv[k][p]);
        const float meanf = cta_sum<DT>(__fadd_rn(sm.x, sm.y), red) * a.inv_n;
        negmean = bc2(-meanf);
        float2 v = bc2(0.f);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            if (t + nt * k < nvec) {
#pragma unroll
                for (int p = 0; p < PW; ++p) {
                    const float2 d = add2(xv[k][p], negmean);
                    v = fma2(d, d, v);
                }
            }
        }
        const float var = cta_sum<DT>(__fadd_rn(v.x, v.y), red) * a.inv_n;
        inv2 = bc2(rsqrtf(var + a.eps));
    }
    const float2 one = bc2(1.0f);
    const float2 nmi = mul2(negmean, inv2);
    const int64_t batch = (KIND >= kAdaLn) ? int64_t(a.tdiv.div(uint32_t(r))) : 0;
    char *yr = reinterpret_cast<char *>(a.y) + r * int64_t(row_bytes);
    const char *scp = reinterpret_cast<const char *>(a.scale) + batch * a.n * ES;
    const char *shp = reinterpret_cast<const char *>(a.shift) + batch * a.n * ES;
    const char *gp = reinterpret_cast<const char *>(a.gate) + batch * a.n * ES;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int j = t + nt * k;
        if (j >= nvec) continue;
        float2 o[PW];
        if (KIND <= kLnMod) {
            float2 wv[PW], bv[PW];
#pragma unroll
            for (int q = 0; q < PW; q += 2) {
                const uint4 wq = a.w ? ld_param(a.w + j * W + 2 * q) : as_u4(make_float4(1.f, 1.f, 1.f, 1.f));
                const uint4 bq = a.b ? ld_param(a.b + j * W + 2 * q) : make_uint4(0, 0, 0, 0);
                unpack2<VOX_CUDA_F32>(wq, wv + q);
                unpack2<VOX_CUDA_F32>(bq, bv + q);
            }
#pragma unroll
            for (int p = 0; p < PW; ++p) {
                if (KIND == kRms) {
                    o[p] = mul2(wv[p], mul2(xv[k][p], inv2));  // kernels.cpp:711, CPU rounding
                } else {
                    const float2 nrm = fma2(xv[k][p], inv2, nmi);
                    if (KIND == kLnMod) o[p] = fma2(add2(one, wv[p]), nrm, bv[p]);  // nn.cpp:262
                    else if (a.w) o[p] = fma2(nrm, wv[p], bv[p]);               // kernels.cpp:722
                    else o[p] = a.b ? add2(nrm, bv[p]) : nrm;
                }
            }
        } else {
            float2 sc[PW], sh[PW], gv[PW], rv[PW];
            unpack2<DT>(ld_param(scp + j * 16), sc);
            unpack2<DT>(ld_param(shp + j * 16), sh);
            if (KIND == kAdaLnGated) {
                unpack2<DT>(ld_param(gp + j * 16), gv);
                unpack2<DT>(rres[k], rv);
            }
#pragma unroll
            for (int p = 0; p < PW; ++p) {
                const float2 nrm = fma2(xv[k][p], inv2, nmi);
                const float2 m = fma2(nrm, add2(one, sc[p]), sh[p]);  // f5.cpp:630
                o[p] = KIND == kAdaLnGated ? fma2(gv[p], m, rv[p]) : m;  // f5.cpp:674
            }
        }
        st_stream(yr + j * 16, pack2<DT>(o));
    }
}

// VOX_CUDA_NORM_CTA: 0 = never take the CTA-per-row path, 1 = always (where it applies); unset = by row count.
int norm_cta_mode() {
    static const int m = [] {
        const char *e = std::getenv("VOX_CUDA_NORM_CTA");
        return e && e[0] == '0' ? 0 : e && e[0] == '1' ? 1 : -1;
    }();
    return m;
}

template <int DT, int KIND, int VPT>
int norm_cta_launch(const NormArgs &a, cudaStream_t st, const char *name) {
    const int64_t nvec = a.n / Vec<DT>::N;
    const int threads = int(((nvec + VPT - 1) / VPT + 31) / 32 * 32);
    launch_k(norm_cta_kernel<DT, KIND, VPT>, dim3(uint32_t(a.rows)), threads, 0, st, a, uint32_t(a.n * (DT == VOX_CUDA_F32 ? 4 : 2)));
    return check_launch(name);
}

// The CTA-per-row path where it applies (few rows, at most 2048 vectors a row), else kPipeNotApplicable.
template <int DT, int KIND>
int norm_cta(const NormArgs &a, cudaStream_t st, const char *name) {
    const int mode = norm_cta_mode();
    const int64_t nvec = a.n / Vec<DT>::N;
    // a warp per row keeps at most rows warps busy: below a quarter of a resident wave of 32-warp SMs, one CTA a row
    const bool few = a.rows <= int64_t(sm_count()) * 8;
    if (mode == 0 || (mode < 0 && !few) || nvec > 2 * kCtaRowMaxThreads || a.rows > 2147483647) return kPipeNotApplicable;
    if (nvec <= kCtaRowMaxThreads) return norm_cta_launch<DT, KIND, 1>(a, st, name);
    return norm_cta_launch<DT, KIND, 2>(a, st, name);
}

template <int DT, int KIND, int VPL>
int norm_pipe_vpl(const NormArgs &a, cudaStream_t st, const char *name) {
    if constexpr (KIND == kAdaLnGated && (DT == VOX_CUDA_F32 ? VPL <= 8 : VPL <= 4)) {  // rows held in registers
        if (adaln_ac_enabled()) {
            const int rc = launch_adaln_ac<DT, VPL>(a, st, name);
            if (rc != kPipeNotApplicable) return rc;
        }
    }
    const uint32_t row_bytes = uint32_t(a.n * (DT == VOX_CUDA_F32 ? 4 : 2));
    const uint32_t stage = KIND == kAdaLnGated ? 2 * row_bytes : row_bytes;
    return launch_row_pipe<NormOp<DT, VPL, KIND>, kStages>(NormOp<DT, VPL, KIND>{a, row_bytes}, a.rows, stage, st, name);
}

template <int DT, int KIND>
int norm_pipe(const NormArgs &a, cudaStream_t st, const char *name) {
    const int rc = norm_cta<DT, KIND>(a, st, name);
    if (rc != kPipeNotApplicable) return rc;
    constexpr int W = Vec<DT>::N;
    const int64_t nvec = a.n / W;
    const int vpl = int((nvec + 31) / 32);
    if (vpl <= 1) return norm_pipe_vpl<DT, KIND, 1>(a, st, name);
    if (vpl <= 2) return norm_pipe_vpl<DT, KIND, 2>(a, st, name);
    if (vpl <= 4) return norm_pipe_vpl<DT, KIND, 4>(a, st, name);
    if (vpl <= 8) return norm_pipe_vpl<DT, KIND, 8>(a, st, name);
    return norm_pipe_vpl<DT, KIND, 16>(a, st, name);
}

template <int DT>
int norm_pipe_kind(int kind, const NormArgs &a, cudaStream_t st, const char *name) {
    switch (kind) {
        case kRms: return norm_pipe<DT, kRms>(a, st, name);
        case kLn: return norm_pipe<DT, kLn>(a, st, name);
        case kLnMod: return norm_pipe<DT, kLnMod>(a, st, name);
        case kAdaLn: return norm_pipe<DT, kAdaLn>(a, st, name);
        default: return norm_pipe<DT, kAdaLnGated>(a, st, name);
    }
}

template <int DT, int VPL>
int add_rms_pipe_vpl(const AddRmsArgs &a, cudaStream_t st) {
    const uint32_t row_bytes = uint32_t(a.n * (DT == VOX_CUDA_F32 ? 4 : 2));
    return launch_row_pipe<AddRmsOp<DT, VPL>, kStages>(AddRmsOp<DT, VPL>{a, row_bytes}, a.rows, 2 * row_bytes, st,
                                                       "vox_cuda_add_rmsnorm");
}

template <int DT>
int add_rms_pipe(const AddRmsArgs &a, cudaStream_t st) {
    const int vpl = int((a.n / Vec<DT>::N + 31) / 32);
    if (vpl <= 1) return add_rms_pipe_vpl<DT, 1>(a, st);
    if (vpl <= 2) return add_rms_pipe_vpl<DT, 2>(a, st);
    if (vpl <= 4) return add_rms_pipe_vpl<DT, 4>(a, st);
    if (vpl <= 8) return add_rms_pipe_vpl<DT, 8>(a, st);
    return add_rms_pipe_vpl<DT, 16>(a, st);
}

}  // namespace

int launch_norm_pipe(int kind, int dtype, const NormArgs &a, cudaStream_t st, const char *name) {
    const int W = dtype == VOX_CUDA_F32 ? 4 : 8;
    bool ok = a.n % W == 0 && a.n / W <= 32 * 16 && aligned16(a.x) && aligned16(a.y) && (!a.w || aligned16(a.w)) &&
              (!a.b || aligned16(a.b)) && a.rows < (int64_t(1) << 32) && a.T > 0 && a.T < (int64_t(1) << 32);
    if (kind >= kAdaLn) ok = ok && aligned16(a.shift) && aligned16(a.scale);
    if (kind == kAdaLnGated) ok = ok && aligned16(a.gate) && aligned16(a.res);
    if (!ok) return kPipeNotApplicable;
    NormArgs b = a;
    b.tdiv = FastDiv(uint32_t(a.T));
    if (dtype == VOX_CUDA_F32) return norm_pipe_kind<VOX_CUDA_F32>(kind, b, st, name);
    return norm_pipe_kind<VOX_CUDA_BF16>(kind, b, st, name);
}

int launch_add_rms_pipe(int dtype, const AddRmsArgs &a, cudaStream_t st) {
    const int W = dtype == VOX_CUDA_F32 ? 4 : 8;
    const bool ok = a.n % W == 0 && a.n / W <= 32 * 16 && aligned16(a.h) && aligned16(a.d) && aligned16(a.xn) &&
                    aligned16(a.w) && (!a.ls || aligned16(a.ls));
    if (!ok) return kPipeNotApplicable;
    if (dtype == VOX_CUDA_F32) return add_rms_pipe<VOX_CUDA_F32>(a, st);
    return add_rms_pipe<VOX_CUDA_BF16>(a, st);
}

int launch_reduce_pipe(const void *x, float *out, int64_t rows, int64_t n, int op, int dtype, cudaStream_t st) {
    const int W = dtype == VOX_CUDA_F32 ? 4 : 8;
    const int64_t row_bytes = n * (dtype == VOX_CUDA_F32 ? 4 : 2);
    // staged rows of up to 16 KB (two stages for each of the CTA's warps stay within the shared memory of one SM)
    if (!(n % W == 0 && row_bytes <= 16384 && aligned16(x))) return kPipeNotApplicable;
    if (dtype == VOX_CUDA_F32) {
        if (op == VOX_CUDA_REDUCE_SUM) return reduce_pipe<VOX_CUDA_F32, VOX_CUDA_REDUCE_SUM>(x, out, rows, n, st);
        if (op == VOX_CUDA_REDUCE_MAX) return reduce_pipe<VOX_CUDA_F32, VOX_CUDA_REDUCE_MAX>(x, out, rows, n, st);
        return reduce_pipe<VOX_CUDA_F32, VOX_CUDA_REDUCE_L2>(x, out, rows, n, st);
    }
    if (op == VOX_CUDA_REDUCE_SUM) return reduce_pipe<VOX_CUDA_BF16, VOX_CUDA_REDUCE_SUM>(x, out, rows, n, st);
    if (op == VOX_CUDA_REDUCE_MAX) return reduce_pipe<VOX_CUDA_BF16, VOX_CUDA_REDUCE_MAX>(x, out, rows, n, st);
    return reduce_pipe<VOX_CUDA_BF16, VOX_CUDA_REDUCE_L2>(x, out, rows, n, st);
}

int launch_softmax_pipe(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len, int64_t pos0, cudaStream_t st) {
    const int64_t nvec = n / 4;
    if (!(n % 4 == 0 && nvec <= 32 * 16 && aligned16(x) && aligned16(y) && rows < (int64_t(1) << 32) && q_len < (int64_t(1) << 32)))
        return kPipeNotApplicable;
    const FastDiv qdiv(uint32_t(q_len > 0 ? q_len : 1));
    const int vpl = int((nvec + 31) / 32);
    const uint32_t stage = uint32_t(n * 4);
    const char *name = "vox_cuda_softmax_rows";
    const bool fold = scale > 0.f && scale <= 3.4e38f;  // positive and finite
    if (vpl <= 1) return fold ? launch_row_pipe<SoftmaxOp<1, true>, kStages>(SoftmaxOp<1, true>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name)
                              : launch_row_pipe<SoftmaxOp<1>, kStages>(SoftmaxOp<1>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name);
    if (vpl <= 2) return fold ? launch_row_pipe<SoftmaxOp<2, true>, kStages>(SoftmaxOp<2, true>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name)
                              : launch_row_pipe<SoftmaxOp<2>, kStages>(SoftmaxOp<2>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name);
    if (vpl <= 4) return fold ? launch_row_pipe<SoftmaxOp<4, true>, kStages>(SoftmaxOp<4, true>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name)
                              : launch_row_pipe<SoftmaxOp<4>, kStages>(SoftmaxOp<4>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name);
    if (vpl <= 8) return fold ? launch_row_pipe<SoftmaxOp<8, true>, kStages>(SoftmaxOp<8, true>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name)
                              : launch_row_pipe<SoftmaxOp<8>, kStages>(SoftmaxOp<8>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name);
    return fold ? launch_row_pipe<SoftmaxOp<16, true>, kStages>(SoftmaxOp<16, true>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name)
                       : launch_row_pipe<SoftmaxOp<16>, kStages>(SoftmaxOp<16>{x, y, n, q_len, pos0, scale, qdiv}, rows, stage, st, name);
}

}  // namespace voxcuda

using namespace voxcuda;

extern "C" int vox_cuda_test_row_stall(int64_t row, uint64_t wait_limit_ns) {
    VOX_REQUIRE(row >= -1, "vox_cuda_test_row_stall: row must be >= -1");
    if (set_wait_test_hook(row, wait_limit_ns) != VOX_CUDA_OK) return check_launch("vox_cuda_test_row_stall");
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_device_error(unsigned int *flags) {
    VOX_REQUIRE(flags != nullptr, "vox_cuda_device_error: flags is NULL");
    unsigned int v = 0;
    if (take_device_error(&v) != VOX_CUDA_OK || gemv_take_device_error(&v) != VOX_CUDA_OK || f5_take_device_error(&v) != VOX_CUDA_OK ||
        gemm_take_device_error(&v) != VOX_CUDA_OK) {
        const cudaError_t e = cudaGetLastError();
        return set_error(VOX_CUDA_ERR_DEVICE, std::string("vox_cuda_device_error: ") + cudaGetErrorString(e));
    }
    *flags = v;
    return VOX_CUDA_OK;
}
