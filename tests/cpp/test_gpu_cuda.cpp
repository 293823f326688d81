// C++ test of the host seam (include/vox_gpu_cuda.hpp): every call goes through the C ABI into the sm_100a kernels
// and is checked against the oracle (oracle/vox_oracle.c, linked as libvox_oracle.so). Built and run by
// tests/test_cpp_host.py on a GPU machine; prints "OK" and exits 0 when every check holds.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "vox_gpu_cuda.hpp"

extern "C" {
void vo_fill(float *out, int64_t n, int dist, float a, float b, uint64_t seed, uint32_t sid, int64_t c0);
void vo_fill_i8(int8_t *out, int64_t n, int a, int b, uint64_t seed, uint32_t sid, int64_t c0);
void vo_fill_u8(uint8_t *out, int64_t n, uint64_t seed, uint32_t sid, int64_t c0);
void vo_rmsnorm_rows(const float *x, const float *w, int64_t rows, int64_t n, float eps, float *out);
void vo_layernorm_rows(const float *x, const float *w, const float *b, int64_t rows, int64_t n, float eps, int modulate, float *out);
void vo_softmax_rows(const float *x, float *y, int64_t rows, int64_t n, float scale, int64_t q_len, int64_t pos0);
void vo_dequant_q8(const int8_t *q, const float *scale, int64_t rows, int64_t cols, float *out);
void vo_dequant_q4(const uint8_t *q, const float *scale, int64_t rows, int64_t cols, float *out);
void vo_snake(const float *x, const float *alpha, const float *beta, float *y, int64_t n, int64_t C, int64_t inner, int kind);
void vo_row_reduce_ordered(const float *x, float *out, int64_t rows, int64_t n, int op, int W);
void vo_rope_inv_freq(int64_t hd, double theta, float *out);
void vo_rope_table(const float *inv_freq, int64_t half, int64_t pos0, int64_t m, float *cs);
void vo_qkv_rope(const float *qkv, const float *qn, const float *kn, const float *cs, float *q, float *kc, float *vc, int64_t m,
                 int64_t heads, int64_t kv_heads, int64_t hd, int64_t pos0, int64_t ring, float eps);
void vo_add_rmsnorm(float *h, const float *d, const float *ls, const float *w, float *xn, int64_t rows, int64_t n, float eps);
void vo_gemv(int q4, const uint8_t *q, const float *scale, const float *bias, const float *x, float *y, double *bound, int64_t rows,
             int64_t cols, int64_t m, int accumulate);
}

static int g_fail = 0;
#define CHECK(c)                                                           \
    do {                                                                   \
        if (!(c)) {                                                        \
            ++g_fail;                                                      \
            std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #c); \
        }                                                                  \
    } while (0)

// |a - b| <= tol * max(|b|, row RMS of b) for every element (rows of n)
static bool close(const std::vector<float> &a, const std::vector<float> &b, int64_t n, double tol) {
    for (size_t r = 0; r * n < b.size(); ++r) {
        double ss = 0;
        for (int64_t i = 0; i < n; ++i) ss += double(b[r * n + i]) * b[r * n + i];
        const double rms = std::sqrt(ss / double(n));
        for (int64_t i = 0; i < n; ++i) {
            const double d = std::fabs(double(a[r * n + i]) - b[r * n + i]);
            if (d > tol * std::max(std::fabs(double(b[r * n + i])), rms)) return false;
        }
    }
    return true;
}
static bool bitexact(const std::vector<float> &a, const std::vector<float> &b) {
    return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * 4) == 0;
}

int main() {
    std::string err;
    if (!vox::gpu_cuda_init(0, err)) {
        std::fprintf(stderr, "init: %s\n", err.c_str());
        return 2;
    }
    std::printf("device: %s\n", vox::gpu_cuda_device_name().c_str());

    // rmsnorm through the host convenience (copy in, run, copy out)
    const int64_t R = 64, N = 1024;
    std::vector<float> x(R * N), w(N), y(R * N), want(R * N);
    vo_fill(x.data(), R * N, 1, 0.f, 1.f, 0, 1, 0);
    vo_fill(w.data(), N, 1, 1.f, 0.02f, 0, 2, 0);
    CHECK(vox::rmsnorm_host(x.data(), w.data(), R, N, 1e-6f, y.data()));
    vo_rmsnorm_rows(x.data(), w.data(), R, N, 1e-6f, want.data());
    CHECK(close(y, want, N, 1e-5));

    // causal softmax [2 heads][64 q][64 k]
    std::vector<float> s(2 * 64 * 64), p(s.size()), ps(s.size());
    vo_fill(s.data(), int64_t(s.size()), 1, 0.f, 3.f, 0, 3, 0);
    CHECK(vox::softmax_causal_host(s.data(), p.data(), 2, 64, 64, 0.0883883f));
    vo_softmax_rows(s.data(), ps.data(), 128, 64, 0.0883883f, 64, 0);
    CHECK(close(p, ps, 64, 1e-5));
    bool zeros = true;
    for (int h = 0; h < 2; ++h)
        for (int q = 0; q < 64; ++q)
            for (int k = q + 1; k < 64; ++k) zeros = zeros && p[(h * 64 + q) * 64 + k] == 0.f;
    CHECK(zeros);

    // q8 / q4 dequantisation: bit-exact with mat_row
    const int64_t QR = 32, QC = 256;
    std::vector<int8_t> q8(QR * QC);
    std::vector<uint8_t> q4(QR * QC / 2);
    std::vector<float> sc(QR * QC / 32), d8(QR * QC), d8w(QR * QC), d4(QR * QC), d4w(QR * QC);
    vo_fill_i8(q8.data(), QR * QC, -128, 127, 0, 4, 0);
    vo_fill_u8(q4.data(), QR * QC / 2, 0, 5, 0);
    vo_fill(sc.data(), int64_t(sc.size()), 0, 0.001f, 0.05f, 0, 6, 0);
    CHECK(vox::dequant_host(false, q8.data(), sc.data(), QR, QC, d8.data()));
    CHECK(vox::dequant_host(true, q4.data(), sc.data(), QR, QC, d4.data()));
    vo_dequant_q8(q8.data(), sc.data(), QR, QC, d8w.data());
    vo_dequant_q4(q4.data(), sc.data(), QR, QC, d4w.data());
    CHECK(bitexact(d8, d8w));
    CHECK(bitexact(d4, d4w));

    // device-pointer calls: LayerNorm (modulate form), Kokoro Snake (bit-exact), row sum (bit-exact order)
    float *dx = static_cast<float *>(vox::gpu_cuda_alloc(R * N * 4)), *dy = static_cast<float *>(vox::gpu_cuda_alloc(R * N * 4));
    float *dw = static_cast<float *>(vox::gpu_cuda_alloc(N * 4)), *db = static_cast<float *>(vox::gpu_cuda_alloc(N * 4));
    float *dr = static_cast<float *>(vox::gpu_cuda_alloc(R * 4));
    CHECK(dx && dy && dw && db && dr);
    std::vector<float> b(N);
    vo_fill(b.data(), N, 1, 0.f, 0.1f, 0, 7, 0);
    CHECK(vox::gpu_cuda_upload(dx, x.data(), R * N * 4) && vox::gpu_cuda_upload(dw, w.data(), N * 4) &&
          vox::gpu_cuda_upload(db, b.data(), N * 4));
    CHECK(vox::gpu_layernorm(dx, dw, db, R, N, 1e-5f, dy));
    CHECK(vox::gpu_cuda_download(y.data(), dy, R * N * 4) && vox::gpu_cuda_sync());
    vo_layernorm_rows(x.data(), w.data(), b.data(), R, N, 1e-5f, 0, want.data());
    CHECK(close(y, want, N, 1e-5));

    std::vector<float> alpha(16);
    vo_fill(alpha.data(), 16, 0, 0.2f, 2.0f, 0, 8, 0);
    CHECK(vox::gpu_cuda_upload(dw, alpha.data(), 16 * 4));
    CHECK(vox::gpu_snake(dx, dw, nullptr, dy, R * N, 16, 1, VOX_CUDA_SNAKE_KOKORO));  // time-major [T][16]
    CHECK(vox::gpu_cuda_download(y.data(), dy, R * N * 4) && vox::gpu_cuda_sync());
    vo_snake(x.data(), alpha.data(), nullptr, want.data(), R * N, 16, 1, 2);
    CHECK(bitexact(y, want));

    std::vector<float> rs(R), rsw(R);
    CHECK(vox::gpu_row_reduce(dx, dr, R, N, VOX_CUDA_REDUCE_SUM));
    CHECK(vox::gpu_cuda_download(rs.data(), dr, R * 4) && vox::gpu_cuda_sync());
    vo_row_reduce_ordered(x.data(), rsw.data(), R, N, 0, 4);
    CHECK(bitexact(rs, rsw));

    // transformer chain: split + RoPE + cache write (bit-exact with the host table, no head norm), residual + RMSNorm
    {
        const int64_t m = 3, nh = 2, nkv = 1, hd = 128, pos0 = 5, W = (nh + 2 * nkv) * hd;
        std::vector<float> qkv(m * W), inv(hd / 2), cs(m * hd), q(m * nh * hd), kc(8 * nkv * hd, 0.f), vc(8 * nkv * hd, 0.f);
        std::vector<float> wq(q.size()), wk(kc.size(), 0.f), wv(vc.size(), 0.f);
        vo_fill(qkv.data(), m * W, 1, 0.f, 1.f, 0, 9, 0);
        vo_rope_inv_freq(hd, 1e6, inv.data());
        vo_rope_table(inv.data(), hd / 2, pos0, m, cs.data());
        float *dq = static_cast<float *>(vox::gpu_cuda_alloc(m * W * 4)), *dcs = static_cast<float *>(vox::gpu_cuda_alloc(cs.size() * 4));
        float *dqo = static_cast<float *>(vox::gpu_cuda_alloc(q.size() * 4)), *dk = static_cast<float *>(vox::gpu_cuda_alloc(kc.size() * 4));
        float *dv = static_cast<float *>(vox::gpu_cuda_alloc(vc.size() * 4));
        CHECK(dq && dcs && dqo && dk && dv);
        CHECK(vox::gpu_cuda_upload(dq, qkv.data(), m * W * 4) && vox::gpu_cuda_upload(dcs, cs.data(), cs.size() * 4) &&
              vox::gpu_cuda_upload(dk, kc.data(), kc.size() * 4) && vox::gpu_cuda_upload(dv, vc.data(), vc.size() * 4));
        CHECK(vox::gpu_qkv_rope(dq, nullptr, nullptr, dcs, dqo, dk, dv, m, nh, nkv, hd, pos0, 1e-6f));
        CHECK(vox::gpu_cuda_download(q.data(), dqo, q.size() * 4) && vox::gpu_cuda_download(kc.data(), dk, kc.size() * 4) &&
              vox::gpu_cuda_download(vc.data(), dv, vc.size() * 4) && vox::gpu_cuda_sync());
        vo_qkv_rope(qkv.data(), nullptr, nullptr, cs.data(), wq.data(), wk.data(), wv.data(), m, nh, nkv, hd, pos0, 0, 1e-6f);
        CHECK(bitexact(q, wq) && bitexact(kc, wk) && bitexact(vc, wv));
        for (void *ptr : {static_cast<void *>(dq), static_cast<void *>(dcs), static_cast<void *>(dqo), static_cast<void *>(dk),
                          static_cast<void *>(dv)})
            vox::gpu_cuda_free(ptr);

        std::vector<float> h0(x), d(R * N), hw(x), xw(R * N), hg(R * N), xg(R * N);
        vo_fill(d.data(), R * N, 1, 0.f, 1.f, 0, 10, 0);
        CHECK(vox::gpu_cuda_upload(dx, h0.data(), R * N * 4) && vox::gpu_cuda_upload(dy, d.data(), R * N * 4) &&
              vox::gpu_cuda_upload(dw, w.data(), N * 4));
        float *dxn = static_cast<float *>(vox::gpu_cuda_alloc(R * N * 4));
        CHECK(dxn && vox::gpu_add_rmsnorm(dx, dy, nullptr, dw, dxn, R, N, 1e-6f));
        CHECK(vox::gpu_cuda_download(hg.data(), dx, R * N * 4) && vox::gpu_cuda_download(xg.data(), dxn, R * N * 4) &&
              vox::gpu_cuda_sync());
        vo_add_rmsnorm(hw.data(), d.data(), nullptr, w.data(), xw.data(), R, N, 1e-6f);
        CHECK(bitexact(hg, hw) && close(xg, xw, N, 1e-5));
        vox::gpu_cuda_free(dxn);
    }

    // decode matvec, Q8 with f32 scales: |y - exact| <= 1e-6 * sum |w x|
    {
        const int64_t GR = 300, GC = 512, M = 2;
        std::vector<int8_t> gq(GR * GC);
        std::vector<float> gs(GR * GC / 32), gx(M * GC), gy(M * GR), gw(M * GR);
        std::vector<double> bound(M * GR);
        vo_fill_i8(gq.data(), GR * GC, -128, 127, 0, 11, 0);
        vo_fill(gs.data(), int64_t(gs.size()), 0, 0.001f, 0.05f, 0, 12, 0);
        vo_fill(gx.data(), M * GC, 1, 0.f, 1.f, 0, 13, 0);
        void *dgq = vox::gpu_cuda_alloc(gq.size()), *dgs = vox::gpu_cuda_alloc(gs.size() * 4);
        float *dgx = static_cast<float *>(vox::gpu_cuda_alloc(gx.size() * 4)), *dgy = static_cast<float *>(vox::gpu_cuda_alloc(gy.size() * 4));
        CHECK(dgq && dgs && dgx && dgy);
        CHECK(vox::gpu_cuda_upload(dgq, gq.data(), gq.size()) && vox::gpu_cuda_upload(dgs, gs.data(), gs.size() * 4) &&
              vox::gpu_cuda_upload(dgx, gx.data(), gx.size() * 4));
        CHECK(vox::gpu_matvec(false, dgq, dgs, VOX_CUDA_F32, nullptr, dgx, dgy, GR, GC, M));
        CHECK(vox::gpu_cuda_download(gy.data(), dgy, gy.size() * 4) && vox::gpu_cuda_sync());
        vo_gemv(0, reinterpret_cast<const uint8_t *>(gq.data()), gs.data(), nullptr, gx.data(), gw.data(), bound.data(), GR, GC, M, 0);
        bool ok = true;
        for (size_t i = 0; i < gy.size(); ++i) ok = ok && std::fabs(double(gy[i]) - gw[i]) <= 1e-6 * bound[i] + 1e-30;
        CHECK(ok);
        for (void *ptr : {dgq, dgs, static_cast<void *>(dgx), static_cast<void *>(dgy)}) vox::gpu_cuda_free(ptr);
    }

    // a rejected call returns false and leaves its reason in the stats, as the Vulkan seam does
    const auto before = vox::gpu_cuda_stats();
    CHECK(!vox::gpu_rmsnorm(dx, dw, R, 0, 1e-6f, dy));
    const auto after = vox::gpu_cuda_stats();
    CHECK(after.calls_failed == before.calls_failed + 1);
    CHECK(after.last_error.find("bad shape") != std::string::npos);

    for (void *ptr : {static_cast<void *>(dx), static_cast<void *>(dy), static_cast<void *>(dw), static_cast<void *>(db),
                      static_cast<void *>(dr)})
        vox::gpu_cuda_free(ptr);
    if (g_fail) {
        std::fprintf(stderr, "%d check(s) failed\n", g_fail);
        return 1;
    }
    std::printf("OK (%lld calls)\n", (long long)vox::gpu_cuda_stats().calls_ok);
    return 0;
}
