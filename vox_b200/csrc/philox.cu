// Seeded synthetic inputs on the device with Vox's counter-based generator, so that multi-GB benchmark tensors
// are produced where they are used (each shard draws its own counters; no host->device broadcast of data).
//
// Philox4x32-10 with Vox's constants and round structure (sampling.hpp:16-33): 10 rounds, key bumped by
// (0x9E3779B9, 0xBB67AE85) between rounds. DetRng::uniform (sampling.hpp:43-46): counter {i lo, i hi, stream, draw},
// key {seed lo, seed hi}, u = (r0 >> 8) * 2^-24. Normal numbers: Box–Muller on element pairs as F5Model::noise
// (f5.cpp:402-414), in f64, then rounded to f32.
#include <math.h>

#include "common.cuh"

namespace voxcuda {
namespace {

struct U4 {
    uint32_t a, b, c, d;
};

__device__ __forceinline__ U4 philox_round(U4 c, uint32_t k0, uint32_t k1) {
    const uint64_t p0 = uint64_t(0xD2511F53u) * c.a, p1 = uint64_t(0xCD9E8D57u) * c.c;
    return U4{uint32_t(p1 >> 32) ^ c.b ^ k0, uint32_t(p1), uint32_t(p0 >> 32) ^ c.d ^ k1, uint32_t(p0)};
}

__device__ __forceinline__ U4 philox10(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int i = 0; i < 10; ++i) {
        c = philox_round(c, k0, k1);
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

__device__ __forceinline__ float det_uniform(uint64_t frame, uint32_t stream, uint32_t draw, uint64_t seed) {
    const U4 r = philox10(U4{uint32_t(frame), uint32_t(frame >> 32), stream, draw}, uint32_t(seed), uint32_t(seed >> 32));
    return float(r.a >> 8) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(256) fill_kernel(void *out, int64_t n, int dist, float a, float b, uint64_t seed, uint32_t sid,
                                                   int64_t c0, int dtype) {
    pdl_enter();
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t g = uint64_t(c0 + i);
        if (dist == 3) {
            const U4 r = philox10(U4{uint32_t(g), uint32_t(g >> 32), sid, 0u}, uint32_t(seed), uint32_t(seed >> 32));
            reinterpret_cast<uint8_t *>(out)[i] = uint8_t(r.a & 0xFFu);
            continue;
        }
        if (dist == 2) {
            const float u = det_uniform(g, sid, 0, seed);
            const int span = int(b) - int(a) + 1;
            int v = int(floorf(u * float(span))) + int(a);
            v = v > int(b) ? int(b) : v;
            reinterpret_cast<int8_t *>(out)[i] = int8_t(v);
            continue;
        }
        float v;
        if (dist == 0) {
            v = __fadd_rn(a, __fmul_rn(__fsub_rn(b, a), det_uniform(g, sid, 0, seed)));
        } else {
            const uint64_t p = g >> 1;
            const double u1 = double(det_uniform(p, sid, 0, seed)), u2 = double(det_uniform(p, sid, 1, seed));
            const double r = sqrt(-2.0 * log(1.0 - u1));
            const double ang = 2.0 * 3.14159265358979323846 * u2;
            const float z = float((g & 1) ? r * sin(ang) : r * cos(ang));
            v = __fadd_rn(a, __fmul_rn(b, z));
        }
        if (dtype == VOX_CUDA_BF16) reinterpret_cast<uint16_t *>(out)[i] = to_bf16(v);
        else reinterpret_cast<float *>(out)[i] = v;
    }
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" int vox_cuda_fill_philox(void *out, int64_t n, int dist, float a, float b, uint64_t seed, uint32_t stream_id,
                                    int64_t counter0, int dtype, void *stream) {
    VOX_REQUIRE(dist >= 0 && dist <= 3, "vox_cuda_fill_philox: unknown distribution");
    VOX_REQUIRE(dist >= 2 || is_act_dtype(dtype), "vox_cuda_fill_philox: dtype must be F32 or BF16");
    VOX_REQUIRE(dist != 2 || (a >= -128.f && b <= 127.f && a <= b), "vox_cuda_fill_philox: integer range must fit int8");
    VOX_REQUIRE(n >= 0 && counter0 >= 0, "vox_cuda_fill_philox: bad size");
    if (n == 0) return VOX_CUDA_OK;
    VOX_REQUIRE(out != nullptr, "vox_cuda_fill_philox: out is NULL");
    const int g = grid_for(n, 256, 16);
    launch_k(fill_kernel, g, 256, 0, reinterpret_cast<cudaStream_t>(stream), out, n, dist, a, b, seed, stream_id, counter0, dtype);
    return check_launch("vox_cuda_fill_philox");
}
