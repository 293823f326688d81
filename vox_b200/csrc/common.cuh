// Shared device helpers and host-side launch plumbing of the vox_cuda library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/vox_cuda.h"

namespace voxcuda {

// ------------------------------------------------------------------ host: status and last error

// Stores msg as this thread's last error and returns status (negative).
int set_error(int status, const std::string &msg);
// Checks cudaGetLastError() after a launch; returns VOX_CUDA_OK or VOX_CUDA_ERR_DEVICE with the message set.
int check_launch(const char *what);

// Number of SMs of the current device (cached per device).
int sm_count();
// Maximum dynamic shared memory per block (opt-in) of the current device (cached per device).
int smem_optin();

// Grid size for a grid-stride kernel of `threads` per block that needs `work_items` thread iterations:
// at most `per_sm` blocks on every SM, at least 1.
int grid_for(int64_t work_items, int threads, int per_sm);

// Blocks of `kernel` (with `threads` threads and `smem` dynamic shared memory) resident on the whole device at once
// (occupancy query, cached per kernel and device).
int resident_blocks(const void *kernel, int threads, size_t smem);

// Balanced persistent grid: `units` work units, `per_block` of them taken by one block per pass; the grid is at most
// one resident wave and every block makes the same number of passes (but the last ones), so no block is left
// working alone at the end.
int balanced_grid(int64_t units, int64_t per_block, int resident);

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool is_act_dtype(int d) { return d == VOX_CUDA_F32 || d == VOX_CUDA_BF16; }
inline int dtype_size(int d) { return d == VOX_CUDA_F32 ? 4 : 2; }

// Programmatic dependent launch: every kernel of the library is launched with programmatic stream serialization and
// starts with pdl_enter(), so the next kernel in the stream is scheduled while this one's last blocks drain, and it
// touches no memory before the previous grid has completed (griddepcontrol.wait). Stream order is unchanged.
// VOX_CUDA_PDL=0 in the environment launches without the attribute.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, args...);  // errors are read by check_launch()
}

#define VOX_REQUIRE(cond, msg)                                         \
    do {                                                               \
        if (!(cond)) return ::voxcuda::set_error(VOX_CUDA_ERR_ARG, msg); \
    } while (0)

// ------------------------------------------------------------------ integer division by an invariant divisor

// Unsigned 32-bit division by a divisor fixed at launch (Granlund–Montgomery, round-up multiplier):
// s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1, n / d = (umulhi(n, m) + n) >> s, exact for all n < 2^32.
struct FastDiv {
    uint32_t d, m, s;
    FastDiv() : d(1), m(1), s(0) {}
    explicit FastDiv(uint32_t dv) : d(dv) {
        s = 0;
        while ((uint64_t(1) << s) < uint64_t(dv)) ++s;
        m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << s) - dv)) / dv + 1);
    }
    __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
#if defined(__CUDA_ARCH__)
        const uint32_t t = __umulhi(n, m);
#else
        const uint32_t t = uint32_t((uint64_t(n) * m) >> 32);
#endif
        return uint32_t((uint64_t(t) + n) >> s);
    }
    __host__ __device__ __forceinline__ uint32_t mod(uint32_t n) const { return n - div(n) * d; }
};

// ------------------------------------------------------------------ device: launch order

// Waits for the previous grid of the stream (and its memory). The next grid may be scheduled as this grid's blocks
// exit (a block's exit counts as its trigger); blocks do not trigger earlier, so waiting blocks of the next grid never
// sit beside this grid's working blocks.
__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ device: conversions

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// Round-to-nearest-even f32 -> bf16 pair packed into one word (lo in bits 0..15). For finite values this equals
// the integer rounding (u + 0x7FFF + ((u >> 16) & 1)) >> 16 of python/vox/build.py:94-97.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ uint16_t to_bf16(float v) {
    __nv_bfloat16 b = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t *>(&b);
}
__device__ __forceinline__ float from_bf16(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }

// ------------------------------------------------------------------ device: streaming memory access

// 16-byte load through the read-only path without L1 allocation (data read once).
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
// 16-byte read-only load through L1 (parameters reused by many rows).
__device__ __forceinline__ uint4 ld_param(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
// 16-byte read-only load through L1 that the compiler keeps in program order relative to the other ordered
// accesses (used where hoisting every parameter load of an unrolled loop would cost more registers than it saves).
__device__ __forceinline__ uint4 ld_param_ordered(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
// 8-byte streaming load.
__device__ __forceinline__ uint2 ld_stream8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
// 16-byte store, streaming (evict-first) in L2.
__device__ __forceinline__ void st_stream(void *p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
// 16-byte load through the coherent path (for buffers the same kernel may also write, e.g. y == x).
__device__ __forceinline__ uint4 ld_cg(const void *p) { return __ldcg(reinterpret_cast<const uint4 *>(p)); }

__device__ __forceinline__ float4 as_f4(uint4 v) {
    return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}
__device__ __forceinline__ uint4 as_u4(float4 v) {
    return make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w));
}

// 8 values of a 16-byte vector (4 f32 words hold 4 values; 4 bf16x2 words hold 8 values).
template <int DT> struct Vec;
template <> struct Vec<VOX_CUDA_F32> {
    static constexpr int N = 4;
    __device__ __forceinline__ static void unpack(uint4 v, float *f) {
        f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y); f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
    }
    __device__ __forceinline__ static uint4 pack(const float *f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
    __device__ __forceinline__ static float load1(const void *p, int64_t i) { return reinterpret_cast<const float *>(p)[i]; }
    __device__ __forceinline__ static void store1(void *p, int64_t i, float v) { reinterpret_cast<float *>(p)[i] = v; }
};
template <> struct Vec<VOX_CUDA_BF16> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void unpack(uint4 v, float *f) {
        f[0] = bf16lo(v.x); f[1] = bf16hi(v.x); f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
        f[4] = bf16lo(v.z); f[5] = bf16hi(v.z); f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
    }
    __device__ __forceinline__ static uint4 pack(const float *f) {
        return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
    }
    __device__ __forceinline__ static float load1(const void *p, int64_t i) {
        return from_bf16(reinterpret_cast<const uint16_t *>(p)[i]);
    }
    __device__ __forceinline__ static void store1(void *p, int64_t i, float v) { reinterpret_cast<uint16_t *>(p)[i] = to_bf16(v); }
};

// ------------------------------------------------------------------ device: packed f32x2 arithmetic
// Blackwell issues two f32 lanes per instruction (FADD2 / FMUL2 / FFMA2); each lane is rounded as the scalar
// __fadd_rn / __fmul_rn / __fmaf_rn. The compiler may fuse an FMUL2 into a following FADD2 (one rounding instead
// of two), so code that must keep the CPU's two roundings bit-exactly uses the scalar intrinsics instead.

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 bc2(float v) { return make_float2(v, v); }

// The 16-byte vector of Vec<DT> as W/2 float pairs.
template <int DT> __device__ __forceinline__ void unpack2(uint4 v, float2 *p);
template <> __device__ __forceinline__ void unpack2<VOX_CUDA_F32>(uint4 v, float2 *p) {
    p[0] = make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
    p[1] = make_float2(__uint_as_float(v.z), __uint_as_float(v.w));
}
template <> __device__ __forceinline__ void unpack2<VOX_CUDA_BF16>(uint4 v, float2 *p) {
    p[0] = make_float2(bf16lo(v.x), bf16hi(v.x));
    p[1] = make_float2(bf16lo(v.y), bf16hi(v.y));
    p[2] = make_float2(bf16lo(v.z), bf16hi(v.z));
    p[3] = make_float2(bf16lo(v.w), bf16hi(v.w));
}
template <int DT> __device__ __forceinline__ uint4 pack2(const float2 *p);
template <> __device__ __forceinline__ uint4 pack2<VOX_CUDA_F32>(const float2 *p) {
    return make_uint4(__float_as_uint(p[0].x), __float_as_uint(p[0].y), __float_as_uint(p[1].x), __float_as_uint(p[1].y));
}
template <> __device__ __forceinline__ uint4 pack2<VOX_CUDA_BF16>(const float2 *p) {
    return make_uint4(pack_bf16(p[0].x, p[0].y), pack_bf16(p[1].x, p[1].y), pack_bf16(p[2].x, p[2].y), pack_bf16(p[3].x, p[3].y));
}

// ------------------------------------------------------------------ device: warp reductions (fixed xor butterfly)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace voxcuda
