// ref_shim.cpp — TEST INFRASTRUCTURE, not product code.
//
// Links dariumi/Vox's own CPU operators, compiled from the reference sources where they lie (src/kernels.cpp,
// src/nn.cpp, src/f5.cpp and the few files they need), into oracle/_ref/libvox_ref.so and exposes them with
// extern "C" entry points, batched over rows and over Vox's own thread pool (vox::parallel_for) with Vox's own
// grain sizes. It serves two purposes:
//   1. pin the C restatement (vox_oracle.c) and generate the golden fixtures under tests/golden/;
//   2. time the reference's CPU path on the host cores (bench.py --impl reference, the cpu_baseline leg).
// Where Vox's code is not externally linkable (anonymous-namespace lambdas: the F5 modulate / gated_add, the Snake
// loops) the loop is restated here, around the reference's own helpers (vox::nn::fast_sin, vox::silu, ...), with
// the reference's grain, and cited.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include "f5.hpp"
#include "kernels.hpp"
#include "nn.hpp"
#include "sampling.hpp"

namespace vox {
// resources.cpp (which owns release_pages) is not linked: the mmap helpers that reference it are never called here.
void release_pages(const void *, size_t) {}
}  // namespace vox

using namespace vox;

#define VR_API extern "C" __attribute__((visibility("default")))

VR_API void vr_set_threads(int n) { set_num_threads(n); }
VR_API int vr_num_threads() { return num_threads(); }

// ---------------------------------------------------------------- generator (sampling.hpp, f5.cpp:402-414)

VR_API void vr_philox_block(const uint32_t c[4], const uint32_t k[2], uint32_t out[4]) {
    auto r = Philox4x32::block({c[0], c[1], c[2], c[3]}, {k[0], k[1]});
    for (int i = 0; i < 4; ++i) out[i] = r[size_t(i)];
}
VR_API float vr_uniform(uint64_t seed, uint64_t frame, uint32_t codebook, uint32_t draw) {
    return DetRng(seed).uniform(frame, codebook, draw);
}
VR_API void vr_f5_noise(uint64_t seed, uint32_t chunk, int64_t n, float *out) { F5Model::noise(seed, chunk, size_t(n), out); }

VR_API float vr_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
VR_API float vr_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }

// ---------------------------------------------------------------- normalisation

// vox::rmsnorm (kernels.cpp:707-712) per row: serially, as transformer_forward calls it (kernels.cpp:793), or over
// parallel_for(rows, 16).
VR_API void vr_rmsnorm_rows(const float *x, const float *w, int64_t rows, int64_t n, float eps, float *out, int par) {
    if (!par) {
        for (int64_t r = 0; r < rows; ++r) rmsnorm(x + r * n, w, n, eps, out + r * n);
        return;
    }
    parallel_for(rows, 16, [&](int64_t a, int64_t b) {
        for (int64_t r = a; r < b; ++r) rmsnorm(x + r * n, w, n, eps, out + r * n);
    });
}

// vox::layernorm (kernels.cpp:714-723) per row over parallel_for(rows, 16), as ln_rows (f5.cpp:101-106).
VR_API void vr_layernorm_rows(const float *x, const float *w, const float *b, int64_t rows, int64_t n, float eps, float *out) {
    parallel_for(rows, 16, [&](int64_t a, int64_t e) {
        for (int64_t r = a; r < e; ++r) layernorm(x + r * n, w, b, n, eps, out + r * n);
    });
}

// vox::nn::layer_norm (nn.cpp:248-265), in place.
VR_API void vr_nn_layer_norm(float *x, int T, int C, const float *w, const float *b, float eps, int modulate) {
    nn::layer_norm(x, T, C, w, b, eps, modulate != 0);
}

// F5 adaLN: the modulate lambda (f5.cpp:617-632, parallel_for(R, 16)) then the gated_add lambda (f5.cpp:670-676,
// parallel_for(R, 32)) with src = the modulated rows, per batch b of x [B][T][D]. Restated (lambdas).
VR_API void vr_adaln(const float *x, const float *shift, const float *scale, const float *gate, const float *res, int64_t B,
                     int64_t T, int64_t D, float *out) {
    for (int64_t bb = 0; bb < B; ++bb) {
        const float *sc = scale + bb * D, *sh = shift + bb * D;
        const float *src = x + bb * T * D;
        float *dst = out + bb * T * D;
        parallel_for(T, 16, [&](int64_t r0, int64_t r1) {
            for (int64_t r = r0; r < r1; ++r) {
                const float *xr = src + size_t(r) * size_t(D);
                double mean = 0;
                for (int i = 0; i < D; ++i) mean += xr[i];
                mean /= D;
                double var = 0;
                for (int i = 0; i < D; ++i) { const double dd = xr[i] - mean; var += dd * dd; }
                var /= D;
                const float inv = float(1.0 / std::sqrt(var + 1e-6));
                float *yr = dst + size_t(r) * size_t(D);
                for (int i = 0; i < D; ++i) yr[i] = (xr[i] - float(mean)) * inv * (1.0f + sc[i]) + sh[i];
            }
        });
        if (gate) {
            const float *g = gate + bb * D, *rb = res + bb * T * D;
            parallel_for(T, 32, [&](int64_t r0, int64_t r1) {
                for (int64_t r = r0; r < r1; ++r)
                    for (int i = 0; i < D; ++i) {
                        const float m = dst[size_t(r) * size_t(D) + size_t(i)];
                        dst[size_t(r) * size_t(D) + size_t(i)] = rb[size_t(r) * size_t(D) + size_t(i)];
                        dst[size_t(r) * size_t(D) + size_t(i)] += g[i] * m;
                    }
            });
        }
    }
}

// Broadcast bias-add over parallel_for(T, 64): the loop of vox::nn::linear (nn.cpp:148-155).
VR_API void vr_bias_add(float *y, const float *b, int64_t T, int64_t O) {
    parallel_for(T, 64, [&](int64_t a, int64_t e) {
        for (int64_t t = a; t < e; ++t)
            for (int64_t o = 0; o < O; ++o) y[t * O + o] += b[size_t(o)];
    });
}

// ---------------------------------------------------------------- softmax

// Causal composition of transformer_forward (kernels.cpp:812-819) around vox::softmax_inplace (fast = 0) or
// vox::nn::softmax_fast (fast = 1), over parallel_for(rows, 8) (the F5 attention grain, f5.cpp:650).
VR_API void vr_softmax_rows(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len, int64_t pos0, int fast) {
    parallel_for(rows, 8, [&](int64_t a, int64_t e) {
        for (int64_t r = a; r < e; ++r) {
            int64_t vis = n;
            if (q_len > 0) vis = std::min<int64_t>(n, (r % q_len) + pos0 + 1);
            float *yr = y + r * n;
            for (int64_t j = 0; j < vis; ++j) yr[j] = scale * x[r * n + j];
            if (fast) nn::softmax_fast(yr, vis);
            else softmax_inplace(yr, vis);
            for (int64_t j = vis; j < n; ++j) yr[j] = 0.0f;
        }
    });
}

// ---------------------------------------------------------------- activations

// g[i] = silu(g[i]) * u[i] (kernels.cpp:836) over parallel_for(n, 4096) (the map_inplace grain, nn.hpp:111).
VR_API void vr_silu_mul(const float *g, const float *u, float *h, int64_t n) {
    parallel_for(n, 4096, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) h[i] = silu(g[i]) * u[i];
    });
}
VR_API void vr_gelu_erf(const float *x, float *y, int64_t n) {
    parallel_for(n, 4096, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) y[i] = gelu_erf(x[i]);
    });
}
// vox::nn::gelu_inplace (nn.cpp:87-96): the AVX2 erfc-polynomial path, parallel_for(n, 8192).
VR_API void vr_gelu_inplace(float *x, int64_t n) { nn::gelu_inplace(x, n); }
// F5 gelu_tanh (f5.cpp:93-96), restated (anonymous namespace), over parallel_for(n, 4096).
VR_API void vr_gelu_tanh(const float *x, float *y, int64_t n) {
    parallel_for(n, 4096, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) {
            const float k = 0.7978845608028654f, v = x[i];
            y[i] = 0.5f * v * (1.0f + std::tanh(k * (v + 0.044715f * v * v * v)));
        }
    });
}
VR_API void vr_add(const float *a, const float *b, float *y, int64_t n) {
    parallel_for(n, 4096, [&](int64_t s, int64_t e) {
        for (int64_t i = s; i < e; ++i) y[i] = a[i] + b[i];
    });
}
VR_API void vr_mul(const float *a, const float *b, float *y, int64_t n) {
    parallel_for(n, 4096, [&](int64_t s, int64_t e) {
        for (int64_t i = s; i < e; ++i) y[i] = a[i] * b[i];
    });
}
// Vox's own fast_sin (nn.hpp:26-40), linked from the header.
VR_API float vr_fast_sin(float x) { return nn::fast_sin(x); }

// Snake, channel of element i = (i / inner) % C (inner = 1: Vox's [T][C] layout; inner = T: channel-major [B][C][T]).
// kind 0 HiFT (cosyvoice.cpp:239-248), 1 SnakeBeta (qwen3.cpp:86-94, a / inv_b given), 2 Kokoro (kokoro.cpp:233-242).
// Restated loops (anonymous namespaces), reference helpers. Vox splits its [T][C] tensor as parallel_for(T, 256)
// (cosyvoice.cpp:241, kokoro.cpp:235): a task is 256 time steps of all C channels, 256 C elements. The same task size
// is kept for either layout by splitting the flat element range with a grain of 256 C elements, so a channel-major
// tensor is spread over all threads along time as Vox spreads its own.
VR_API void vr_snake(const float *x, const float *alpha, const float *beta, float *y, int64_t n, int64_t C, int64_t inner, int kind) {
    parallel_for(n, 256 * C, [&](int64_t a, int64_t e) {
        for (int64_t i = a; i < e;) {
            const int64_t c = (i / inner) % C;
            const int64_t stop = std::min(e, (i / inner + 1) * inner);  // end of this channel's run
            const float al = alpha[c];
            if (kind == 0) {
                for (; i < stop; ++i) {
                    const float v = x[i], sn = std::sin(al * v);
                    y[i] = v + (1.0f / (al + 1e-9f)) * (sn * sn);
                }
            } else if (kind == 1) {
                const float bt = beta[c];
                for (; i < stop; ++i) {
                    const float v = x[i], sn = std::sin(v * al);
                    y[i] = v + bt * sn * sn;
                }
            } else {
                for (; i < stop; ++i) {
                    const float v = x[i], sv = nn::fast_sin(al * v);
                    y[i] = v + (1.0f / al) * (sv * sv);
                }
            }
        }
    });
}

// ---------------------------------------------------------------- block dequantisation

// vox::mat_gather (kernels.cpp:468-471) of every row of a Q8 (type 3) or Q4 (type 4) Mat, over parallel_for(rows, 16)
// (the dequant grain of matmul, kernels.cpp:665); f32 scales [rows][cols/32].
VR_API void vr_mat_rows(int type, const uint8_t *data, const float *scale, int64_t rows, int64_t cols, float *out) {
    Mat M;
    M.type = type == 4 ? WType::Q4 : WType::Q8;
    M.data = data;
    M.scale = scale;
    M.rows = rows;
    M.cols = cols;
    parallel_for(rows, 16, [&](int64_t a, int64_t b) {
        for (int64_t r = a; r < b; ++r) mat_gather(M, r, out + r * cols);
    });
}

VR_API void vr_quantize_q8(const float *w, int64_t rows, int64_t cols, int8_t *q, float *scale) {
    std::vector<int8_t> qq;
    std::vector<float> ss;
    quantize_q8(w, rows, cols, qq, ss);
    std::memcpy(q, qq.data(), qq.size());
    std::memcpy(scale, ss.data(), ss.size() * 4);
}
VR_API void vr_quantize_q4(const float *w, int64_t rows, int64_t cols, uint8_t *q, float *scale) {
    std::vector<uint8_t> qq;
    std::vector<float> ss;
    quantize_q4(w, rows, cols, qq, ss);
    std::memcpy(q, qq.data(), qq.size());
    std::memcpy(scale, ss.data(), ss.size() * 4);
}

// ---------------------------------------------------------------- reductions (CPU baseline only)

// Row sum / max / L2 over parallel_for(rows, 16), float accumulation in element order as inside vox::rmsnorm
// (kernels.cpp:709) and softmax_inplace (kernels.cpp:727-729).
VR_API void vr_row_reduce(const float *x, float *out, int64_t rows, int64_t n, int op) {
    parallel_for(rows, 16, [&](int64_t a, int64_t b) {
        for (int64_t r = a; r < b; ++r) {
            const float *xr = x + r * n;
            float acc = op == 1 ? -INFINITY : 0.f;
            for (int64_t i = 0; i < n; ++i) acc = op == 1 ? std::max(acc, xr[i]) : op == 2 ? acc + xr[i] * xr[i] : acc + xr[i];
            out[r] = op == 2 ? std::sqrt(acc) : acc;
        }
    });
}

// ---------------------------------------------------------------- transformer elementwise chain

VR_API void vr_rope_inv_freq(int64_t hd, double theta, float *out) {
    const std::vector<float> f = rope_inv_freq(hd, theta);
    std::memcpy(out, f.data(), f.size() * sizeof(float));
}

// The per-token q/k step of transformer_forward (kernels.cpp:797-803) on the split projections q [m][nh*hd] and
// k [m][nkv*hd], in place: vox::rmsnorm per head (qn / kn may be NULL), then vox::rope_apply at position pos0 + i.
// Restated loop (it lives inside transformer_forward) around the reference's own rmsnorm and rope_apply.
VR_API void vr_qk_norm_rope(float *q, float *k, const float *qn, const float *kn, const float *inv_freq, int64_t m, int64_t nh,
                            int64_t nkv, int64_t hd, int64_t pos0, float eps) {
    const int64_t qd = nh * hd, kd = nkv * hd;
    for (int64_t i = 0; i < m; ++i) {
        float *qi = q + i * qd, *ki = k + i * kd;
        if (qn) for (int64_t hh = 0; hh < nh; ++hh) rmsnorm(qi + hh * hd, qn, hd, eps, qi + hh * hd);
        if (kn) for (int64_t hh = 0; hh < nkv; ++hh) rmsnorm(ki + hh * hd, kn, hd, eps, ki + hh * hd);
        rope_apply(qi, nh, hd, inv_freq, pos0 + i);
        rope_apply(ki, nkv, hd, inv_freq, pos0 + i);
    }
}

// The residual update before an RMSNorm (kernels.cpp:822-825: o *= attn_scale, h += o; then :833) with the
// reference's own rmsnorm per row. ls may be NULL (no layer scale).
VR_API void vr_add_rmsnorm(float *h, const float *d, const float *ls, const float *w, float *xn, int64_t rows, int64_t n, float eps) {
    std::vector<float> o(d, d + rows * n);
    if (ls) for (int64_t i = 0; i < rows; ++i) for (int64_t e = 0; e < n; ++e) o[size_t(i * n + e)] *= ls[e];
    for (int64_t i = 0; i < rows * n; ++i) h[i] += o[size_t(i)];
    for (int64_t i = 0; i < rows; ++i) rmsnorm(h + i * n, w, n, eps, xn + i * n);
}

// ---------------------------------------------------------------- matmul (quantized weights)

// vox::matmul (kernels.cpp:656-706) on a CPU Mat: type 0 = F32, 3 = Q8, 4 = Q4 (WType order), bias may be NULL.
// y[i][r] for i < m. With Q8 and m > 8 this is the dequantise-then-f32 path (kernels.cpp:669-688); with F32 weights
// (e.g. dequantised by mat_rows) the float-activation product of the GPU matvec.
VR_API void vr_matmul(int type, const uint8_t *data, const float *scale, const float *bias, int64_t rows, int64_t cols,
                      const float *x, int64_t m, float *y) {
    Mat W;
    W.type = WType(type);
    W.data = data;
    W.scale = scale;
    W.rows = rows;
    W.cols = cols;
    W.bias = bias;
    matmul(W, x, m, y);
}

// ---------------------------------------------------------------- .tmod container (formats.cpp)

// vox::tmod_write (formats.cpp:215-249) of `count` blobs; manifest_json is the manifest without its "blobs" table.
// dtypes follow DType (common.hpp:22); shapes holds 8 entries per blob, ndims the used ones. 0 on success.
VR_API int vr_tmod_write(const char *path, const char *manifest_json, int64_t count, const char *const *names, const int *dtypes,
                         const int64_t *shapes, const int *ndims, const uint8_t *const *data, const uint64_t *nbytes, uint32_t flags) {
    try {
        std::map<std::string, Tensor> blobs;
        for (int64_t i = 0; i < count; ++i) {
            Tensor t;
            t.dtype = DType(dtypes[i]);
            t.shape.assign(shapes + i * 8, shapes + i * 8 + ndims[i]);
            t.bytes.assign(data[i], data[i] + nbytes[i]);
            blobs.emplace(names[i], std::move(t));
        }
        tmod_write(path, json::parse(manifest_json), blobs, flags);
        return 0;
    } catch (...) {
        return -1;
    }
}

// vox::TmodFile (formats.cpp:175-205): copies blob `name` into out (cap bytes) and returns its size, or -1 (missing
// blob or an exception, e.g. a bad file).
VR_API int64_t vr_tmod_read(const char *path, const char *name, uint8_t *out, uint64_t cap) {
    try {
        TmodFile f(path);
        const TensorView &v = f.get(name);
        if (v.nbytes <= cap) std::memcpy(out, v.data, v.nbytes);
        return int64_t(v.nbytes);
    } catch (...) {
        return -1;
    }
}

// ---------------------------------------------------------------- F5 DiT forward (f5.cpp)

// F5Model (f5.cpp:258-393) loaded from the .tmod file `path` on the CPU (gpu = false), then F5Model::time_embed(t)
// (the SiLU'd time embedding every AdaLN reads, f5.cpp:510-526) into ts [dim] and F5Model::dit_forward(B, N, x, cond,
// temb, t) into out [B][N][mel_dim] (f5.cpp:563-724). Returns 0, or -1 with the exception's message in err.
VR_API int vr_f5_dit(const char *path, int B, int N, const float *x, const float *cond, const float *temb, float t, float *ts,
                     float *out, char *err, int errcap) {
    try {
        auto f = std::make_shared<TmodFile>(path);
        F5Model m(f, false);
        std::vector<float> tv;
        m.time_embed(t, tv);
        std::memcpy(ts, tv.data(), tv.size() * sizeof(float));
        m.dit_forward(B, N, x, cond, temb, t, out);
        return 0;
    } catch (const std::exception &e) {
        std::snprintf(err, size_t(errcap), "%s", e.what());
        return -1;
    }
}

// ---------------------------------------------------------------- the CPU arm of the benchmark suite (bench.py)
//
// Out-of-place and bf16-I/O forms of the operators above, so the reference's CPU code runs the GPU suite's own
// workload: same shapes, same element types in memory, outputs preallocated by the caller. Each keeps the reference's
// arithmetic and its parallel_for grain; bf16 values are widened exactly and rounded to nearest-even once at the store
// (python/vox/build.py:94-97). A parallel_for whose range fits one grain runs inline in the calling thread
// (ThreadPool::run, kernels.cpp:56-57), which is how Vox's own in-place operators run on one task's chunk below.

static inline float bf16f(uint16_t h) { return bf16_to_f32(h); }
static inline uint16_t f32bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return uint16_t((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// y = gelu(x) with vox::nn::gelu_inplace (nn.cpp:87-96) on each parallel_for(n, 8192) task's chunk: the chunk is
// copied to y (it stays in cache) and transformed in place there.
VR_API void vr_gelu_f32(const float *x, float *y, int64_t n) {
    parallel_for(n, 8192, [&](int64_t a, int64_t b) {
        std::memcpy(y + a, x + a, size_t(b - a) * sizeof(float));
        nn::gelu_inplace(y + a, b - a);
    });
}
VR_API void vr_gelu_bf16(const uint16_t *x, uint16_t *y, int64_t n) {
    parallel_for(n, 8192, [&](int64_t a, int64_t b) {
        float buf[8192];
        for (int64_t i = a; i < b; ++i) buf[i - a] = bf16f(x[i]);
        nn::gelu_inplace(buf, b - a);
        for (int64_t i = a; i < b; ++i) y[i] = f32bf(buf[i - a]);
    });
}
VR_API void vr_add_bf16(const uint16_t *a, const uint16_t *b, uint16_t *y, int64_t n) {
    parallel_for(n, 4096, [&](int64_t s, int64_t e) {
        for (int64_t i = s; i < e; ++i) y[i] = f32bf(bf16f(a[i]) + bf16f(b[i]));
    });
}
VR_API void vr_mul_bf16(const uint16_t *a, const uint16_t *b, uint16_t *y, int64_t n) {
    parallel_for(n, 4096, [&](int64_t s, int64_t e) {
        for (int64_t i = s; i < e; ++i) y[i] = f32bf(bf16f(a[i]) * bf16f(b[i]));
    });
}
// Row sum / max / L2 of bf16 rows: vr_row_reduce's order on the widened values.
VR_API void vr_row_reduce_bf16(const uint16_t *x, float *out, int64_t rows, int64_t n, int op) {
    parallel_for(rows, 16, [&](int64_t a, int64_t b) {
        for (int64_t r = a; r < b; ++r) {
            const uint16_t *xr = x + r * n;
            float acc = op == 1 ? -INFINITY : 0.f;
            for (int64_t i = 0; i < n; ++i) {
                const float v = bf16f(xr[i]);
                acc = op == 1 ? std::max(acc, v) : op == 2 ? acc + v * v : acc + v;
            }
            out[r] = op == 2 ? std::sqrt(acc) : acc;
        }
    });
}
// Global sum of f32 rows [rows][n] (no reference function): row sums as vr_row_reduce, then 840 slot partials in f64
// (slot s = rows [s rows / 840, (s + 1) rows / 840), in row order) over parallel_for(840, 8), folded in slot order.
// rowsum: caller scratch of `rows` floats; slots: caller scratch of 840 doubles.
VR_API double vr_global_sum(const float *x, int64_t rows, int64_t n, float *rowsum, double *slots) {
    vr_row_reduce(x, rowsum, rows, n, 0);
    parallel_for(840, 8, [&](int64_t a, int64_t b) {
        for (int64_t sl = a; sl < b; ++sl) {
            double acc = 0.0;
            for (int64_t r = sl * rows / 840; r < (sl + 1) * rows / 840; ++r) acc += double(rowsum[r]);
            slots[sl] = acc;
        }
    });
    double t = 0.0;
    for (int s = 0; s < 840; ++s) t += slots[s];
    return t;
}
// Block dequantisation to bf16: vox::mat_gather (kernels.cpp:468-471) of each row into the task's f32 row buffer over
// parallel_for(rows, 16) (kernels.cpp:665), rounded to bf16 at the store.
VR_API void vr_mat_rows_bf16(int type, const uint8_t *data, const float *scale, int64_t rows, int64_t cols, uint16_t *out) {
    Mat M;
    M.type = type == 4 ? WType::Q4 : WType::Q8;
    M.data = data;
    M.scale = scale;
    M.rows = rows;
    M.cols = cols;
    parallel_for(rows, 16, [&](int64_t a, int64_t b) {
        std::vector<float> row(static_cast<size_t>(cols));
        for (int64_t r = a; r < b; ++r) {
            mat_gather(M, r, row.data());
            uint16_t *o = out + r * cols;
            for (int64_t i = 0; i < cols; ++i) o[i] = f32bf(row[size_t(i)]);
        }
    });
}
// The F5 adaLN with bf16 activations: the modulate lambda (f5.cpp:617-632, parallel_for(T, 16)) on the widened x rows
// into the caller's f32 buffer m [T][D], then the gated_add lambda (f5.cpp:670-676, parallel_for(T, 32)) from the
// widened residual, rounded to bf16 at the store; per batch b of x [B][T][D]; shift / scale / gate [B][D] bf16.
VR_API void vr_adaln_bf16(const uint16_t *x, const uint16_t *shift, const uint16_t *scale, const uint16_t *gate, const uint16_t *res,
                          int64_t B, int64_t T, int64_t D, float *m, uint16_t *out) {
    for (int64_t bb = 0; bb < B; ++bb) {
        std::vector<float> sc(static_cast<size_t>(D)), sh(static_cast<size_t>(D)), g(static_cast<size_t>(D));
        for (int64_t i = 0; i < D; ++i) {
            sc[size_t(i)] = bf16f(scale[bb * D + i]);
            sh[size_t(i)] = bf16f(shift[bb * D + i]);
            g[size_t(i)] = bf16f(gate[bb * D + i]);
        }
        const uint16_t *src = x + bb * T * D;
        parallel_for(T, 16, [&](int64_t r0, int64_t r1) {
            for (int64_t r = r0; r < r1; ++r) {
                const uint16_t *xr = src + r * D;
                double mean = 0;
                for (int64_t i = 0; i < D; ++i) mean += bf16f(xr[i]);
                mean /= double(D);
                double var = 0;
                for (int64_t i = 0; i < D; ++i) { const double dd = bf16f(xr[i]) - mean; var += dd * dd; }
                var /= double(D);
                const float inv = float(1.0 / std::sqrt(var + 1e-6));
                float *yr = m + r * D;
                for (int64_t i = 0; i < D; ++i) yr[i] = (bf16f(xr[i]) - float(mean)) * inv * (1.0f + sc[size_t(i)]) + sh[size_t(i)];
            }
        });
        const uint16_t *rb = res + bb * T * D;
        uint16_t *dst = out + bb * T * D;
        parallel_for(T, 32, [&](int64_t r0, int64_t r1) {
            for (int64_t r = r0; r < r1; ++r)
                for (int64_t i = 0; i < D; ++i) {
                    float h = bf16f(rb[r * D + i]);
                    h += g[size_t(i)] * m[r * D + i];
                    dst[r * D + i] = f32bf(h);
                }
        });
    }
}
