// Q8 / Q4 block dequantisation (32 weights per block, one scale per block), to f32 or bf16.
//
// Vox layout (kernels.hpp:42-47): Q8 codes int8 [rows][cols], Q4 codes packed [rows][cols/2] with byte j of a
// 16-byte block holding element j (low nibble) and element j+16 (high nibble); scales [rows][cols/32] f32 (Vox's
// loader, nn.cpp:141-143) or f16 (converted exactly to f32 first). Because cols % 32 == 0 the scale of flat
// element e is simply scale[e / 32].
//
// Value = float(code) * scale (Q8, kernels.cpp:450) or float(int(nibble) - 8) * scale (Q4, kernels.cpp:459-460):
// a single f32 multiply, so the f32 result is bit-identical to vox::mat_row, and the bf16 result is its
// round-to-nearest-even.
//
// Each thread produces one 16-byte output vector per iteration (8 bf16 or 4 f32), so every store instruction of
// a warp writes 512 contiguous bytes; the codes come in as 4- or 8-byte loads, kUnroll iterations in flight.
#include "common.cuh"

namespace voxcuda {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;

template <int SDT>
__device__ __forceinline__ float load_scale(const void *s, int64_t i) {
    if (SDT == VOX_CUDA_F16) return __half2float(__ldg(reinterpret_cast<const __half *>(s) + i));
    return __ldg(reinterpret_cast<const float *>(s) + i);
}

// OPT outputs per thread-iteration: 8 for bf16, 4 for f32 (16 bytes either way).
template <int ODT> struct OutVec {
    static constexpr int OPT = ODT == VOX_CUDA_BF16 ? 8 : 4;
    __device__ __forceinline__ static uint4 pack(const float *v) {
        if (ODT == VOX_CUDA_BF16)
            return make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
        return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
    }
};

// Raw code bytes of output vector v: 8 bytes (OPT = 8) or 4 bytes (OPT = 4, in .x), and the nibble shift for Q4.
template <bool Q4, int OPT>
__device__ __forceinline__ uint2 load_code_word(const uint8_t *q, int64_t v) {
    const int64_t e0 = v * OPT;
    const uint8_t *p = Q4 ? q + (e0 >> 5) * 16 + (e0 & 15) : q + e0;  // Q4: byte j of a block holds elements j, j+16
    if (OPT == 8) return ld_stream8(p);
    return make_uint2(__ldcs(reinterpret_cast<const unsigned int *>(p)), 0u);
}
// Exact int -> float of codes without I2F: a byte b placed under the exponent of 2^23 (word 0x4B0000bb) is the float
// 2^23 + b, so one exact subtraction gives the code. Q8: b = code ^ 0x80 (code + 128), subtract 2^23 + 128.
// Q4: b = nibble (0..15), subtract 2^23 + 8 (the value (u - 8) of kernels.cpp:459-460).
__device__ __forceinline__ float byte_as_float(uint32_t word, uint32_t sel) {
    // selector picks one byte of `word` into bits 0..7, zero bytes 1..2, 0x4B into byte 3
    return __uint_as_float(__byte_perm(word, 0x4B000000u, sel));
}
template <bool Q4, int OPT>
__device__ __forceinline__ void decode(uint2 w, int64_t v, float *c) {
    uint32_t lo, hi;
    if (!Q4) {
        lo = w.x ^ 0x80808080u;
        hi = w.y ^ 0x80808080u;
    } else {
        const int sh = int((v * OPT) & 16) >> 2;  // 0: low nibbles (elements 0..15 of the block), 4: high (16..31)
        lo = (w.x >> sh) & 0x0F0F0F0Fu;
        hi = (w.y >> sh) & 0x0F0F0F0Fu;
    }
    const float2 off = bc2(Q4 ? -8388616.0f : -8388736.0f);
    float2 p[OPT / 2];
    p[0] = add2(make_float2(byte_as_float(lo, 0x7440), byte_as_float(lo, 0x7441)), off);
    p[1] = add2(make_float2(byte_as_float(lo, 0x7442), byte_as_float(lo, 0x7443)), off);
    if (OPT == 8) {
        p[2] = add2(make_float2(byte_as_float(hi, 0x7440), byte_as_float(hi, 0x7441)), off);
        p[3] = add2(make_float2(byte_as_float(hi, 0x7442), byte_as_float(hi, 0x7443)), off);
    }
#pragma unroll
    for (int k = 0; k < OPT / 2; ++k) {
        c[2 * k] = p[k].x;
        c[2 * k + 1] = p[k].y;
    }
}

template <bool Q4, int SDT, int ODT>
__global__ void __launch_bounds__(kThreads) dequant_kernel(const uint8_t *q, const void *scale, void *out, int64_t nvec) {
    pdl_enter();
    constexpr int OPT = OutVec<ODT>::OPT;
    constexpr int VPB = 32 / OPT;  // output vectors per 32-weight block
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    uint4 *po = reinterpret_cast<uint4 *>(out);
    // kUnroll output vectors per thread per iteration, the last iteration predicated (its loads still in flight
    // together); the code words stay packed until they are used
    for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += kUnroll * stride) {
        uint2 cw[kUnroll];
        float s[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t w = v + u * stride;
            if (w < nvec) {
                cw[u] = load_code_word<Q4, OPT>(q, w);
                s[u] = load_scale<SDT>(scale, w / VPB);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t w = v + u * stride;
            if (w < nvec) {
                float c[OPT];
                decode<Q4, OPT>(cw[u], w, c);
                float f[OPT];
                const float2 s2 = bc2(s[u]);
#pragma unroll
                for (int k = 0; k < OPT; k += 2) {
                    const float2 p = mul2(make_float2(c[k], c[k + 1]), s2);  // one rounding each, as kernels.cpp:450,459
                    f[k] = p.x;
                    f[k + 1] = p.y;
                }
                st_stream(po + w, OutVec<ODT>::pack(f));
            }
        }
    }
}

template <bool Q4>
int launch_dequant(const uint8_t *q, const void *scale, int sdt, void *out, int odt, int64_t rows, int64_t cols, void *stream,
                   const char *name) {
    VOX_REQUIRE(sdt == VOX_CUDA_F32 || sdt == VOX_CUDA_F16, std::string(name) + ": scale dtype must be F32 or F16");
    VOX_REQUIRE(odt == VOX_CUDA_F32 || odt == VOX_CUDA_BF16, std::string(name) + ": out dtype must be F32 or BF16");
    VOX_REQUIRE(rows >= 0 && cols >= 0 && cols % 32 == 0, std::string(name) + ": cols must be a multiple of 32");
    const int64_t n = rows * cols;
    if (n == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(q && scale && out, std::string(name) + ": NULL pointer");
    VOX_REQUIRE(aligned16(out), std::string(name) + ": out must be 16-byte aligned");
    VOX_REQUIRE((reinterpret_cast<uintptr_t>(q) & 7u) == 0, std::string(name) + ": codes must be 8-byte aligned");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int opt = odt == VOX_CUDA_BF16 ? 8 : 4;
    const int64_t nvec = n / opt;
    auto kern = odt == VOX_CUDA_BF16 ? (sdt == VOX_CUDA_F16 ? dequant_kernel<Q4, VOX_CUDA_F16, VOX_CUDA_BF16> : dequant_kernel<Q4, VOX_CUDA_F32, VOX_CUDA_BF16>)
                                     : (sdt == VOX_CUDA_F16 ? dequant_kernel<Q4, VOX_CUDA_F16, VOX_CUDA_F32> : dequant_kernel<Q4, VOX_CUDA_F32, VOX_CUDA_F32>);
    const int g = balanced_grid(nvec, int64_t(kThreads) * kUnroll, resident_blocks((const void *)kern, kThreads, 0));
    launch_k(kern, g, kThreads, 0, st, q, scale, out, nvec);
    return check_launch(name);
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_dequant_q8(const int8_t *q, const void *scale, int scale_dtype, void *out, int out_dtype, int64_t rows, int64_t cols,
                        void *stream) {
    return launch_dequant<false>(reinterpret_cast<const uint8_t *>(q), scale, scale_dtype, out, out_dtype, rows, cols, stream,
                                 "vox_cuda_dequant_q8");
}

int vox_cuda_dequant_q4(const uint8_t *q, const void *scale, int scale_dtype, void *out, int out_dtype, int64_t rows, int64_t cols,
                        void *stream) {
    return launch_dequant<true>(q, scale, scale_dtype, out, out_dtype, rows, cols, stream, "vox_cuda_dequant_q4");
}

}  // extern "C"
