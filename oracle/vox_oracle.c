/*
 * vox_oracle.c — TEST INFRASTRUCTURE, not product code.
 *
 * A plain-C restatement of dariumi/Vox's CPU arithmetic for the memory-bound operator path (src/kernels.cpp,
 * src/nn.cpp, src/nn.hpp, src/f5.cpp, src/qwen3.cpp, src/cosyvoice.cpp, src/kokoro.cpp, src/sampling.hpp,
 * python/vox/build.py). It is the parity oracle of the CUDA kernels: only the tests, the smoke check and the CPU
 * baseline leg of bench.py load it. Every function cites the reference lines it restates. The library is built
 * with -ffp-contract=off so that each float multiply and add is rounded as in Vox's baseline x86-64 build, and it
 * calls glibc's expf/erff/tanhf/sinf/sqrtf exactly where Vox calls std::exp/erf/tanh/sin/sqrt on floats.
 *
 * The restatement is pinned against the reference itself: oracle/ref_shim.cpp compiles Vox's own kernels.cpp,
 * nn.cpp (and f5.cpp for the noise generator) from their sources into oracle/_ref/libvox_ref.so, and
 * tests/golden/make_golden.py records that library's outputs as committed fixtures.
 *
 * All functions take host pointers, row-major, and are batched over rows where Vox works one row per call.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define VO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------ generator: sampling.hpp:16-50, f5.cpp:402-414 */

/* Philox4x32-10 block (sampling.hpp:19-32). */
VO_API void vo_philox_block(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
    for (int i = 0; i < 10; ++i) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n1 = (uint32_t)p1, n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1, n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        if (i < 9) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

static uint32_t philox_r0(uint64_t seed, uint64_t frame, uint32_t codebook, uint32_t draw) {
    const uint32_t c[4] = {(uint32_t)frame, (uint32_t)(frame >> 32), codebook, draw};
    const uint32_t k[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t r[4];
    vo_philox_block(c, k, r);
    return r[0];
}

/* DetRng::uniform (sampling.hpp:43-46): 24-bit uniform in [0, 1). */
VO_API float vo_uniform(uint64_t seed, uint64_t frame, uint32_t codebook, uint32_t draw) {
    return (float)(philox_r0(seed, frame, codebook, draw) >> 8) * (1.0f / 16777216.0f);
}

/* Box–Muller of F5Model::noise (f5.cpp:405-411) for element g of a stream. */
static float normal_elem(uint64_t seed, uint32_t sid, uint64_t g) {
    const uint64_t p = g >> 1;
    const double u1 = (double)vo_uniform(seed, p, sid, 0), u2 = (double)vo_uniform(seed, p, sid, 1);
    const double r = sqrt(-2.0 * log(1.0 - u1));
    const double a = 2.0 * 3.14159265358979323846 * u2;
    return (float)((g & 1) ? r * sin(a) : r * cos(a));
}

/* The synthetic inputs of the benchmark (same definition as vox_cuda_fill_philox): dist 0 uniform [a, b),
 * dist 1 normal(a, b). Element i uses counter index c0 + i. */
VO_API void vo_fill(float *out, int64_t n, int dist, float a, float b, uint64_t seed, uint32_t sid, int64_t c0) {
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t g = (uint64_t)(c0 + i);
        if (dist == 0) out[i] = a + (b - a) * vo_uniform(seed, g, sid, 0);
        else out[i] = a + b * normal_elem(seed, sid, g);
    }
}
/* Integer codes uniform in [a, b] (dist 2) and raw bytes (dist 3) of vox_cuda_fill_philox. */
VO_API void vo_fill_i8(int8_t *out, int64_t n, int a, int b, uint64_t seed, uint32_t sid, int64_t c0) {
    for (int64_t i = 0; i < n; ++i) {
        const float u = vo_uniform(seed, (uint64_t)(c0 + i), sid, 0);
        int v = (int)floorf(u * (float)(b - a + 1)) + a;
        out[i] = (int8_t)(v > b ? b : v);
    }
}
VO_API void vo_fill_u8(uint8_t *out, int64_t n, uint64_t seed, uint32_t sid, int64_t c0) {
    for (int64_t i = 0; i < n; ++i) out[i] = (uint8_t)(philox_r0(seed, (uint64_t)(c0 + i), sid, 0) & 0xFFu);
}

/* F5Model::noise (f5.cpp:402-414) for n values of chunk `chunk`: stream 0xF5000000 + chunk. */
VO_API void vo_f5_noise(uint64_t seed, uint32_t chunk, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = normal_elem(seed, 0xF5000000u + chunk, (uint64_t)i);
}

/* ------------------------------------------------------------ half precision: kernels.hpp:63-76, build.py:94-97 */

VO_API float vo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (ex == 0) {
        if (man == 0) bits = sign;
        else {
            int e = -1;
            do { ++e; man <<= 1; } while (!(man & 0x400u));
            bits = sign | (uint32_t)(127 - 15 - e) << 23 | (man & 0x3FFu) << 13;
        }
    } else if (ex == 31) bits = sign | 0x7F800000u | man << 13;
    else bits = sign | (ex + 112) << 23 | man << 13;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}
VO_API float vo_bf16_to_f32(uint16_t h) {
    const uint32_t b = (uint32_t)h << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}
/* python/vox/build.py:94-97: (u + 0x7FFF + ((u >> 16) & 1)) >> 16 */
VO_API uint16_t vo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
VO_API void vo_f32_to_bf16_n(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = vo_f32_to_bf16(x[i]);
}
VO_API void vo_f16_to_f32_n(const uint16_t *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = vo_f16_to_f32(x[i]);
}

/* ------------------------------------------------------------ normalisation */

/* vox::rmsnorm (kernels.cpp:707-712), one call per row. */
VO_API void vo_rmsnorm_rows(const float *x, const float *w, int64_t rows, int64_t n, float eps, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        float *o = out + r * n;
        float ss = 0;
        for (int64_t i = 0; i < n; ++i) ss += xr[i] * xr[i];
        const float inv = 1.0f / sqrtf(ss / (float)n + eps);
        for (int64_t i = 0; i < n; ++i) o[i] = w[i] * (xr[i] * inv);
    }
}

/* vox::layernorm (kernels.cpp:714-723) when modulate = 0 (w NULL: plain normalisation as nn.cpp:262, b NULL: no
 * shift); vox::nn::layer_norm's modulate form (1 + w) * n + b (nn.cpp:259-262) when modulate = 1. */
VO_API void vo_layernorm_rows(const float *x, const float *w, const float *b, int64_t rows, int64_t n, float eps, int modulate,
                              float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        float *o = out + r * n;
        double mean = 0;
        for (int64_t i = 0; i < n; ++i) mean += xr[i];
        mean /= (double)n;
        double var = 0;
        for (int64_t i = 0; i < n; ++i) { const double d = xr[i] - mean; var += d * d; }
        var /= (double)n;
        const float inv = (float)(1.0 / sqrt(var + (double)eps));
        for (int64_t i = 0; i < n; ++i) {
            const float nrm = (xr[i] - (float)mean) * inv;
            if (modulate) o[i] = (1.0f + w[i]) * nrm + b[i];
            else if (w) o[i] = nrm * w[i] + (b ? b[i] : 0.0f);
            else o[i] = b ? nrm + b[i] : nrm;
        }
    }
}

/* F5's modulate lambda (f5.cpp:617-632): LN without affine, eps 1e-6 (a double literal there; `eps` here), then
 * (x - mean) * inv * (1 + sc[i]) + sh[i]. */
VO_API void vo_modulate(const float *x, const float *sc, const float *sh, int64_t rows, int64_t D, double eps, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * D;
        double mean = 0;
        for (int64_t i = 0; i < D; ++i) mean += xr[i];
        mean /= (double)D;
        double var = 0;
        for (int64_t i = 0; i < D; ++i) { const double dd = xr[i] - mean; var += dd * dd; }
        var /= (double)D;
        const float inv = (float)(1.0 / sqrt(var + eps));
        float *yr = out + r * D;
        for (int64_t i = 0; i < D; ++i) yr[i] = (xr[i] - (float)mean) * inv * (1.0f + sc[i]) + sh[i];
    }
}

/* F5's gated_add lambda (f5.cpp:670-676): h[r][i] += gate[i] * src[r][i]. */
VO_API void vo_gated_add(float *h, const float *gate, const float *src, int64_t rows, int64_t D) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t i = 0; i < D; ++i) h[r * D + i] += gate[i] * src[r * D + i];
}

/* The fused adaLN block over x [B][T][D]: per batch b, modulate with shift/scale[b] (f5.cpp:617-632), then, when
 * gate and residual are given, out = residual + gate[b] * m (f5.cpp:670-676 with src = m). */
VO_API void vo_adaln(const float *x, const float *shift, const float *scale, const float *gate, const float *res, int64_t B,
                     int64_t T, int64_t D, double eps, float *out) {
    for (int64_t b = 0; b < B; ++b) {
        float *ob = out + b * T * D;
        vo_modulate(x + b * T * D, scale + b * D, shift + b * D, T, D, eps, ob);
        if (gate) {
            for (int64_t t = 0; t < T; ++t)
                for (int64_t i = 0; i < D; ++i) {
                    const float m = ob[t * D + i];
                    ob[t * D + i] = res[(b * T + t) * D + i];
                    ob[t * D + i] += gate[b * D + i] * m;
                }
        }
    }
}

/* Broadcast bias-add, the loop of vox::nn::linear (nn.cpp:151-154): y[t][o] += b[o]. */
VO_API void vo_bias_add(float *y, const float *b, int64_t rows, int64_t D) {
    for (int64_t t = 0; t < rows; ++t)
        for (int64_t o = 0; o < D; ++o) y[t * D + o] += b[o];
}

/* ------------------------------------------------------------ softmax */

/* vox::softmax_inplace (kernels.cpp:725-732). */
VO_API void vo_softmax_inplace(float *x, int64_t n) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; ++i) mx = x[i] > mx ? x[i] : mx; /* std::max(mx, x[i]) */
    float sum = 0;
    for (int64_t i = 0; i < n; ++i) { x[i] = expf(x[i] - mx); sum += x[i]; }
    const float inv = 1.0f / sum;
    for (int64_t i = 0; i < n; ++i) x[i] *= inv;
}

/* The causal attention-score composition of transformer_forward (kernels.cpp:812-819): row r of [rows][n] is
 * query r % q_len at absolute position pos0 + r % q_len and sees n_vis = min(n, pos0 + r % q_len + 1) keys;
 * sc[j] = scale * x[j], softmax_inplace over those, zeros after. q_len = 0: every row sees all n entries. */
VO_API void vo_softmax_rows(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len, int64_t pos0) {
    for (int64_t r = 0; r < rows; ++r) {
        int64_t vis = n;
        if (q_len > 0) {
            vis = (r % q_len) + pos0 + 1;
            if (vis > n) vis = n;
        }
        float *yr = y + r * n;
        for (int64_t j = 0; j < vis; ++j) yr[j] = scale * x[r * n + j];
        vo_softmax_inplace(yr, vis);
        for (int64_t j = vis; j < n; ++j) yr[j] = 0.0f;
    }
}

/* ------------------------------------------------------------ activations */

/* silu (kernels.hpp:105) in the SwiGLU loop g[i] = silu(g[i]) * u[i] (kernels.cpp:836). */
VO_API void vo_silu_mul(const float *g, const float *u, float *h, int64_t n) {
    for (int64_t i = 0; i < n; ++i) h[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}
/* swiglu.comp:8-12 layout: gu [m][2I] -> h [m][I]. */
VO_API void vo_swiglu_fused(const float *gu, float *h, int64_t m, int64_t I) {
    for (int64_t r = 0; r < m; ++r)
        for (int64_t e = 0; e < I; ++e) {
            const float a = gu[r * 2 * I + e], u = gu[r * 2 * I + I + e];
            h[r * I + e] = (a / (1.0f + expf(-a))) * u;
        }
}
/* gelu_erf (kernels.hpp:106). */
VO_API void vo_gelu_erf(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = 0.5f * x[i] * (1.0f + erff(x[i] * 0.70710678118654752440f));
}
/* F5's gelu_tanh (f5.cpp:93-96). */
VO_API void vo_gelu_tanh(const float *x, float *y, int64_t n) {
    const float k = 0.7978845608028654f;
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i];
        y[i] = 0.5f * v * (1.0f + tanhf(k * (v + 0.044715f * v * v * v)));
    }
}
VO_API void vo_add(const float *a, const float *b, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = a[i] + b[i];
}
VO_API void vo_mul(const float *a, const float *b, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = a[i] * b[i];
}

/* Vox's fast_sin (nn.hpp:26-40). */
VO_API float vo_fast_sin(float x) {
    const float q = nearbyintf(x * 0.31830988618379067f);
    float r = x - q * 3.140625f;
    r = r - q * 9.67502593994140625e-4f;
    r = r - q * 1.509957990978376432e-7f;
    const float r2 = r * r;
    float p = -2.39e-8f;
    p = p * r2 + 2.7526e-6f;
    p = p * r2 - 1.98409e-4f;
    p = p * r2 + 8.3333315e-3f;
    p = p * r2 - 1.6666666e-1f;
    const float s = r + r * r2 * p;
    const int qi = (int)q;
    return (qi & 1) ? -s : s;
}

/* Snake over n elements whose channel is (i / inner) % C. kind 0: HiFT SnakeRes::snake (cosyvoice.cpp:239-248);
 * kind 1: snake_apply with the Snake struct a / inv_b (qwen3.cpp:86-94); kind 2: Kokoro (kokoro.cpp:233-242). */
VO_API void vo_snake(const float *x, const float *alpha, const float *beta, float *y, int64_t n, int64_t C, int64_t inner, int kind) {
    for (int64_t i = 0; i < n; ++i) {
        const int64_t c = (i / inner) % C;
        const float v = x[i];
        if (kind == 0) {
            const float al = alpha[c], sn = sinf(al * v);
            y[i] = v + (1.0f / (al + 1e-9f)) * (sn * sn);
        } else if (kind == 1) {
            const float sn = sinf(v * alpha[c]);
            y[i] = v + beta[c] * sn * sn;
        } else {
            const float s = vo_fast_sin(alpha[c] * v);
            y[i] = v + (1.0f / alpha[c]) * (s * s);
        }
    }
}
/* load_snake (qwen3.cpp:76-84). */
VO_API void vo_load_snake(const float *alpha, const float *beta, float *a, float *inv_b, int64_t C) {
    for (int64_t c = 0; c < C; ++c) {
        a[c] = expf(alpha[c]);
        inv_b[c] = 1.0f / (expf(beta[c]) + 1e-9f);
    }
}

/* ------------------------------------------------------------ block dequantisation: kernels.cpp:446-463 */

/* mat_row Q8: tmp[b*32+j] = float(p[b*32+j]) * s[b]. */
VO_API void vo_dequant_q8(const int8_t *q, const float *scale, int64_t rows, int64_t cols, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const int8_t *p = q + r * cols;
        const float *s = scale + r * (cols / 32);
        for (int64_t b = 0; b < cols / 32; ++b)
            for (int j = 0; j < 32; ++j) out[r * cols + b * 32 + j] = (float)p[b * 32 + j] * s[b];
    }
}
/* mat_row Q4: low nibble of byte j -> element j, high nibble -> element j + 16, value (u - 8) * s[b]. */
VO_API void vo_dequant_q4(const uint8_t *q, const float *scale, int64_t rows, int64_t cols, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const uint8_t *p = q + r * (cols / 2);
        const float *s = scale + r * (cols / 32);
        float *o = out + r * cols;
        for (int64_t b = 0; b < cols / 32; ++b)
            for (int j = 0; j < 16; ++j) {
                const uint8_t v = p[b * 16 + j];
                o[b * 32 + j] = (float)((int)(v & 15) - 8) * s[b];
                o[b * 32 + 16 + j] = (float)((int)(v >> 4) - 8) * s[b];
            }
    }
}

/* ------------------------------------------------------------ reductions (no reference function; see header) */

/* Row sum / max / L2 in the fixed order of the CUDA kernel (vox_cuda.h, vox_cuda_row_reduce): vectors of W
 * elements, lane l takes vectors l, l+32, ..., element k of a vector into accumulator k % 4, lane value
 * (a0 + a1) + (a2 + a3), lanes folded by the xor butterfly 16, 8, 4, 2, 1. op 0 sum, 1 max, 2 L2. */
VO_API void vo_row_reduce_ordered(const float *x, float *out, int64_t rows, int64_t n, int op, int W) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        const int64_t nvec = (n + W - 1) / W;
        float lane[32];
        for (int l = 0; l < 32; ++l) {
            float acc[4];
            for (int k = 0; k < 4; ++k) acc[k] = op == 1 ? -INFINITY : 0.0f;
            for (int64_t j = l; j < nvec; j += 32)
                for (int k = 0; k < W; ++k) {
                    const int64_t e = j * W + k;
                    if (e >= n) continue;
                    const float v = xr[e];
                    if (op == 1) acc[k % 4] = fmaxf(acc[k % 4], v);
                    else if (op == 2) acc[k % 4] = acc[k % 4] + v * v;
                    else acc[k % 4] = acc[k % 4] + v;
                }
            if (op == 1) lane[l] = fmaxf(fmaxf(acc[0], acc[1]), fmaxf(acc[2], acc[3]));
            else lane[l] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        }
        for (int o = 16; o > 0; o >>= 1) {
            float nxt[32];
            for (int l = 0; l < 32; ++l) nxt[l] = op == 1 ? fmaxf(lane[l], lane[l ^ o]) : lane[l] + lane[l ^ o];
            memcpy(lane, nxt, sizeof(lane));
        }
        out[r] = op == 2 ? sqrtf(lane[0]) : lane[0];
    }
}

/* The same reductions in f64, sequential: the accuracy reference. */
VO_API void vo_row_reduce_f64(const float *x, double *out, int64_t rows, int64_t n, int op) {
    for (int64_t r = 0; r < rows; ++r) {
        double acc = op == 1 ? -INFINITY : 0.0;
        for (int64_t i = 0; i < n; ++i) {
            const double v = x[r * n + i];
            if (op == 1) acc = v > acc ? v : acc;
            else if (op == 2) acc += v * v;
            else acc += v;
        }
        out[r] = op == 2 ? sqrt(acc) : acc;
    }
}

#define VO_SLOTS 840
static int64_t slot_begin(int64_t s, int64_t R) { return (s * R) / VO_SLOTS; }

/* Global-sum slot partials of a shard (rows [row0, row0 + rows) of R) from its f32 row sums: owned slot s =
 * f64 sum of row sums lo..hi-1 where lane l adds rows lo+l, lo+l+32, ... and lanes fold by the xor butterfly;
 * other slots 0. Same order as vox_cuda_global_sum_partials. */
VO_API void vo_global_sum_slots(const float *rowsum, int64_t row0, int64_t rows, int64_t R, double *slots) {
    for (int64_t s = 0; s < VO_SLOTS; ++s) {
        const int64_t lo = slot_begin(s, R), hi = slot_begin(s + 1, R);
        if (!(lo >= row0 && hi <= row0 + rows)) { slots[s] = 0.0; continue; }
        double lane[32];
        for (int l = 0; l < 32; ++l) {
            lane[l] = 0.0;
            for (int64_t r = lo + l; r < hi; r += 32) lane[l] += (double)rowsum[r - row0];
        }
        for (int o = 16; o > 0; o >>= 1) {
            double nxt[32];
            for (int l = 0; l < 32; ++l) nxt[l] = lane[l] + lane[l ^ o];
            memcpy(lane, nxt, sizeof(lane));
        }
        slots[s] = lane[0];
    }
}

/* Fold of the 840 slots as vox_cuda_global_sum_finish: thread t of 256 adds slots t, t+256, ... in order; each warp
 * of 32 folds by the xor butterfly; the 8 warp values (padded to 32 with zeros) fold by the butterfly again. */
VO_API double vo_global_sum_finish(const double *slots) {
    double th[256];
    for (int t = 0; t < 256; ++t) {
        th[t] = 0.0;
        for (int s = t; s < VO_SLOTS; s += 256) th[t] += slots[s];
    }
    double wv[32];
    for (int w = 0; w < 8; ++w) {
        double lane[32];
        for (int l = 0; l < 32; ++l) lane[l] = th[w * 32 + l];
        for (int o = 16; o > 0; o >>= 1) {
            double nxt[32];
            for (int l = 0; l < 32; ++l) nxt[l] = lane[l] + lane[l ^ o];
            memcpy(lane, nxt, sizeof(lane));
        }
        wv[w] = lane[0];
    }
    for (int w = 8; w < 32; ++w) wv[w] = 0.0;
    for (int o = 16; o > 0; o >>= 1) {
        double nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = wv[l] + wv[l ^ o];
        memcpy(wv, nxt, sizeof(wv));
    }
    return wv[0];
}

/* ------------------------------------------------------------ transformer elementwise chain (per layer, per token)
 * The non-GEMM steps between a layer's fused QKV projection and its attention, and the residual update before each
 * RMSNorm: kernels.cpp:734-757 (rope_inv_freq, rope_apply), kernels.cpp:793-803 and 822-833 (transformer_forward),
 * shaders/qkvsplit.comp, shaders/qkrope.comp, shaders/ringput.comp and the table of gpu_vulkan.cpp:855-860. */

/* rope_inv_freq (kernels.cpp:734-738): inv_freq[i] = float(1 / theta^(2i / hd)) in double. */
VO_API void vo_rope_inv_freq(int64_t hd, double theta, float *out) {
    for (int64_t i = 0; i < hd / 2; ++i) out[i] = (float)(1.0 / pow(theta, (double)(2 * i) / (double)hd));
}

/* The RoPE table of the GPU transformer (gpu_vulkan.cpp:855-860): row i is position pos0 + i, entry p holds
 * cos(f), sin(f) of f = inv_freq[p] * float(pos0 + i), all in float as rope_apply (kernels.cpp:744-747). */
VO_API void vo_rope_table(const float *inv_freq, int64_t half, int64_t pos0, int64_t m, float *cs) {
    for (int64_t i = 0; i < m; ++i)
        for (int64_t p = 0; p < half; ++p) {
            const float f = inv_freq[p] * (float)(pos0 + i);
            cs[(i * half + p) * 2] = cosf(f);
            cs[(i * half + p) * 2 + 1] = sinf(f);
        }
}

/* vox::rmsnorm (kernels.cpp:707-712) of one head in place, then rope_apply's rotate-half (kernels.cpp:749-756)
 * with the table row cs (half pairs). */
static void head_norm_rope(float *p, const float *nw, const float *cs, int64_t hd, float eps) {
    const int64_t half = hd / 2;
    if (nw) {
        float ss = 0;
        for (int64_t e = 0; e < hd; ++e) ss += p[e] * p[e];
        const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
        for (int64_t e = 0; e < hd; ++e) p[e] = nw[e] * (p[e] * inv);
    }
    for (int64_t i = 0; i < half; ++i) {
        const float c = cs[2 * i], s = cs[2 * i + 1], a = p[i], b = p[i + half];
        p[i] = a * c - b * s;
        p[i + half] = b * c + a * s;
    }
}

/* One layer's QKV split, q/k head RMSNorm and RoPE, and K/V cache write for m tokens at positions pos0 .. pos0+m-1.
 * qkv [m][qd + 2 kd] is the fused projection (qkvsplit.comp:10-19); q [m][qd]; token i's K and V rows go to cache
 * row pos0 + i, or to ring slot (pos0 + i) % ring when ring > 0 (ringput.comp:11). Head norms (qn, kn, either
 * NULL) and the rotation follow transformer_forward (kernels.cpp:797-803); cs holds table rows 0 .. m-1
 * (vo_rope_table). */
VO_API void vo_qkv_rope(const float *qkv, const float *qn, const float *kn, const float *cs, float *q, float *kc, float *vc,
                        int64_t m, int64_t heads, int64_t kv_heads, int64_t hd, int64_t pos0, int64_t ring, float eps) {
    const int64_t qd = heads * hd, kd = kv_heads * hd, w = qd + 2 * kd, half = hd / 2;
    for (int64_t i = 0; i < m; ++i) {
        const float *src = qkv + i * w, *csr = cs + i * half * 2;
        const int64_t slot = ring > 0 ? (pos0 + i) % ring : pos0 + i;
        float *qi = q + i * qd, *ki = kc + slot * kd, *vi = vc + slot * kd;
        memcpy(qi, src, (size_t)qd * 4);
        memcpy(ki, src + qd, (size_t)kd * 4);
        memcpy(vi, src + qd + kd, (size_t)kd * 4);
        for (int64_t h = 0; h < heads; ++h) head_norm_rope(qi + h * hd, qn, csr, hd, eps);
        for (int64_t h = 0; h < kv_heads; ++h) head_norm_rope(ki + h * hd, kn, csr, hd, eps);
    }
}

/* The residual update and the RMSNorm that follows it (kernels.cpp:822-825 then :833; :829-831 then the next
 * layer's :793): d *= ls (the optional per-channel layer scale, attn_scale / mlp_scale), h += d, xn = rmsnorm(h, w)
 * (kernels.cpp:707-712). h is updated in place. */
VO_API void vo_add_rmsnorm(float *h, const float *d, const float *ls, const float *w, float *xn, int64_t rows, int64_t n, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        float *hr = h + r * n;
        const float *dr = d + r * n;
        for (int64_t e = 0; e < n; ++e) hr[e] += ls ? dr[e] * ls[e] : dr[e];
    }
    vo_rmsnorm_rows(h, w, rows, n, eps, xn);
}

/* ------------------------------------------------------------ quantized GEMV (decode, m <= 8)
 * y[i][r] = bias[r] + sum_k W[r][k] * x[i][k] (y[i][r] += ... when accumulate), W[r][k] = q * scale[r][k/32]:
 * the semantics of Vox's GPU matvec shaders/matmul.comp:1-8, 60-178 (float activations, weights dequantized in the
 * shader) and of the CPU matmul's dequantise-then-f32 path (kernels.cpp:669-688). Q8: int8 codes [rows][cols];
 * Q4: 16 bytes per 32-block, byte j = weight j | weight j+16 << 4, value (u - 8) * scale (kernels.hpp:45-47).
 * Accumulated in double; `bound` receives sum_k |W[r][k] x[i][k]| (the scale of a dot product's rounding error). */
VO_API void vo_gemv(int q4, const uint8_t *q, const float *scale, const float *bias, const float *x, float *y, double *bound,
                    int64_t rows, int64_t cols, int64_t m, int accumulate) {
    const int64_t nb = cols / 32;
    for (int64_t i = 0; i < m; ++i)
        for (int64_t r = 0; r < rows; ++r) {
            double s = 0, a = 0;
            for (int64_t k = 0; k < cols; ++k) {
                const int64_t b = k / 32, j = k % 32;
                int v;
                if (q4) {
                    const uint8_t byte = q[r * (cols / 2) + b * 16 + (j & 15)];
                    v = (int)(j < 16 ? (byte & 15) : (byte >> 4)) - 8;
                } else {
                    v = (int8_t)q[r * cols + k];
                }
                const double p = (double)((float)v * scale[r * nb + b]) * (double)x[i * cols + k];
                s += p;
                a += fabs(p);
            }
            const double out = (bias ? (double)bias[r] : 0.0) + s;
            const int64_t o = i * rows + r;
            y[o] = accumulate ? (float)((double)y[o] + out) : (float)out;
            if (bound) bound[o] = a;
        }
}
