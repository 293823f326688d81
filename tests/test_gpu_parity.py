"""GPU parity tests: every sm_100a kernel, called through the C ABI (vox_b200 -> libvox_cuda.so), against the oracle
(the C restatement of Vox's CPU arithmetic, pinned to the reference by the golden fixtures) on the same seeded
inputs.

Bars (north star): bit-exact for q8/q4 dequantisation, integer/byte generation and the fixed-order reductions;
|got - want| <= 1e-5 * max(|want|, row RMS of want) for f32 results; 1e-2 relative (same floor) for bf16 results,
against the oracle run in f32 on the bf16-rounded inputs. Config-size cases use BASELINE's shapes.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_TOL = 1e-2


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.cpu().numpy()


def bf16r(a):
    """Values of a rounded to bf16 (RNE), as f32."""
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def assert_close(got, want, tol=F32_TOL, floor=None):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape
    if floor is None:
        floor = np.sqrt(np.mean(want.reshape(-1, want.shape[-1]) ** 2, axis=-1)).reshape(want.shape[:-1] + (1,)) if want.ndim else 0.0
    bound = tol * np.maximum(np.abs(want), floor) + 1e-30
    bad = np.abs(got - want) > bound
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(f"{bad.sum()} of {bad.size} elements out of tolerance; first at {tuple(i)}: got {got[tuple(i)]!r} "
                             f"want {want[tuple(i)]!r} bound {np.broadcast_to(bound, got.shape)[tuple(i)]!r}")


def assert_bitexact(got, want):
    np.testing.assert_array_equal(np.ascontiguousarray(got, np.float32).view(np.uint32),
                                  np.ascontiguousarray(want, np.float32).view(np.uint32))


def unaligned(a, dtype=None):
    """A device copy of `a` whose data pointer is one element past a 16-byte boundary (scalar kernel path)."""
    t = dev(a) if dtype is None else dev(a, dtype)
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device="cuda")
    v = buf[1:].view(t.shape)
    v.copy_(t)
    assert v.data_ptr() % 16 != 0
    return v


# ------------------------------------------------------------------ generator

def test_fill_philox_matches_oracle(vox, port):
    n = 100003
    u = vox.fill_philox(torch.empty(n, device="cuda"), 0, -1.5, 2.5, seed=5, stream_id=9, counter0=77)
    assert_bitexact(host(u), port.fill(n, 0, -1.5, 2.5, seed=5, sid=9, c0=77))
    z = vox.fill_philox(torch.empty(n, device="cuda"), 1, 0.0, 3.0, seed=5, stream_id=9)
    np.testing.assert_allclose(host(z), port.fill(n, 1, 0.0, 3.0, seed=5, sid=9), rtol=0, atol=3e-6)
    q = vox.fill_philox(torch.empty(n, dtype=torch.int8, device="cuda"), 2, -128, 127, seed=1, stream_id=2)
    np.testing.assert_array_equal(host(q), port.fill_i8((n,), -128, 127, seed=1, sid=2))
    b = vox.fill_philox(torch.empty(n, dtype=torch.uint8, device="cuda"), 3, 0, 0, seed=1, stream_id=3)
    np.testing.assert_array_equal(host(b), port.fill_u8((n,), seed=1, sid=3))


# ------------------------------------------------------------------ normalisation

def test_rmsnorm_golden_and_config(vox, port, golden):
    g = golden["norm"]
    assert_close(host(vox.rmsnorm(dev(g["x"]), dev(g["w"]), 1e-6)), g["rmsnorm"])
    assert_close(host(vox.rmsnorm(dev(g["x33"]), dev(g["w"][:33]), 1e-6)), g["rmsnorm33"])
    # x [512,1024] ~N(0,1), w ~N(1,0.02), eps 1e-6
    x = port.normal((512, 1024))
    w = port.normal((1024,), 1.0, 0.02, sid=1)
    want = port.rmsnorm(x, w, 1e-6)
    out = vox.rmsnorm(dev(x), dev(w), 1e-6)
    assert_close(host(out), want)
    # deterministic run to run, in place, on an unaligned buffer, on another stream
    assert_bitexact(host(vox.rmsnorm(dev(x), dev(w), 1e-6)), host(out))
    xi = dev(x)
    vox.rmsnorm(xi, dev(w), 1e-6, out=xi)
    assert_bitexact(host(xi), host(out))
    xu = unaligned(x)
    assert_close(host(vox.rmsnorm(xu, dev(w), 1e-6, out=unaligned(np.zeros_like(x)))), want)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        o2 = vox.rmsnorm(dev(x), dev(w), 1e-6)
    s.synchronize()
    assert_bitexact(host(o2), host(out))


@pytest.mark.parametrize("n", [1, 7, 32, 100, 2048, 2052, 4096, 8192])
def test_rmsnorm_row_lengths(vox, port, n):
    x = port.normal((37, n), sid=n)
    w = port.normal((n,), 1.0, 0.02, sid=n + 1)
    assert_close(host(vox.rmsnorm(dev(x), dev(w), 1e-6)), port.rmsnorm(x, w, 1e-6))


@pytest.mark.parametrize("rows", [64, 1184, 2000])
@pytest.mark.parametrize("n", [1024, 6144])
def test_norm_kinds_both_row_paths(vox, port, rows, n):
    """Every norm kind, f32 and bf16, at row counts that take the CTA-per-row path (few rows: up to 8 per SM) and
    the warp-per-row pipeline (or, for rows of more than 512 vectors, the general path)."""
    B = 2 if rows % 2 == 0 else 1
    T = rows // B
    x = port.normal((rows, n), 0.3, 1.5, sid=900 + n)
    w = port.normal((n,), 1.0, 0.1, sid=901)
    b = port.normal((n,), 0.0, 0.1, sid=902)
    res = port.normal((rows, n), sid=903)
    sh, sc, g = (port.normal((B, n), 0.0, 0.1, sid=s) for s in (904, 905, 906))
    assert_close(host(vox.rmsnorm(dev(x), dev(w), 1e-6)), port.rmsnorm(x, w, 1e-6))
    assert_close(host(vox.layernorm(dev(x), dev(w), dev(b), 1e-5)), port.layernorm(x, w, b, 1e-5))
    assert_close(host(vox.layernorm(dev(x), dev(w), dev(b), 1e-6, modulate=True)), port.layernorm(x, w, b, 1e-6, modulate=True))
    assert_close(host(vox.layernorm(dev(x), None, None, 1e-6)), port.layernorm(x, None, None, 1e-6))
    X, R = x.reshape(B, T, n), res.reshape(B, T, n)
    assert_close(host(vox.adaln(dev(X), dev(sh), dev(sc), 1e-6)), port.adaln(X, sh, sc))
    assert_close(host(vox.adaln(dev(X), dev(sh), dev(sc), 1e-6, dev(g), dev(R))), port.adaln(X, sh, sc, g, R))
    xb, rb = bf16r(X), bf16r(R)
    shb, scb, gb = bf16r(sh), bf16r(sc), bf16r(g)
    d = lambda a: dev(a, torch.bfloat16)  # noqa: E731
    assert_close(host(vox.rmsnorm(d(xb.reshape(rows, n)), dev(w), 1e-6)), bf16r(port.rmsnorm(xb.reshape(rows, n), w, 1e-6)), BF16_TOL)
    assert_close(host(vox.adaln(d(xb), d(shb), d(scb), 1e-6, d(gb), d(rb))), bf16r(port.adaln(xb, shb, scb, gb, rb)), BF16_TOL)
    # in place (y = x) and y = residual
    xi = dev(X)
    vox.adaln(xi, dev(sh), dev(sc), 1e-6, dev(g), dev(R), out=xi)
    assert_close(host(xi), port.adaln(X, sh, sc, g, R))
    ri = dev(R)
    vox.adaln(dev(X), dev(sh), dev(sc), 1e-6, dev(g), ri, out=ri)
    assert_close(host(ri), port.adaln(X, sh, sc, g, R))


def test_rmsnorm_bf16(vox, port):
    x = bf16r(port.normal((64, 1024), sid=3))
    w = port.normal((1024,), 1.0, 0.02, sid=4)
    want = bf16r(port.rmsnorm(x, w, 1e-6))
    assert_close(host(vox.rmsnorm(dev(x, torch.bfloat16), dev(w), 1e-6)), want, BF16_TOL)


def test_layernorm_golden(vox, golden):
    g = golden["norm"]
    x, w, b = dev(g["x"]), dev(g["w"]), dev(g["b"])
    assert_close(host(vox.layernorm(x, w, b, 1e-5)), g["layernorm"])
    assert_close(host(vox.layernorm(x, w, None, 1e-5)), g["layernorm_nob"])
    assert_close(host(vox.layernorm(x, w, b, 1e-6, modulate=True)), g["ln_modulate"])
    assert_close(host(vox.layernorm(x, None, None, 1e-6)), g["ln_plain"])


@pytest.mark.parametrize("n", [5, 1024, 3000, 6144])
def test_layernorm_shapes_and_bf16(vox, port, n):
    x = port.normal((19, n), 0.5, 2.0, sid=n)
    w = port.normal((n,), 1.0, 0.1, sid=n + 1)
    b = port.normal((n,), 0.0, 0.1, sid=n + 2)
    assert_close(host(vox.layernorm(dev(x), dev(w), dev(b), 1e-5)), port.layernorm(x, w, b, 1e-5))
    xb = bf16r(x)
    assert_close(host(vox.layernorm(dev(xb, torch.bfloat16), dev(w), dev(b), 1e-6, modulate=True)),
                 bf16r(port.layernorm(xb, w, b, 1e-6, modulate=True)), BF16_TOL)
    y = vox.layer_norm(dev(x), dev(w), dev(b), 1e-5)  # in place
    assert_close(host(y), port.layernorm(x, w, b, 1e-5))


def test_adaln_golden(vox, golden):
    g = golden["norm"]
    assert_close(host(vox.adaln(dev(g["X"]), dev(g["shift"]), dev(g["scale"]), 1e-6, dev(g["gate"]), dev(g["res"]))),
                 g["adaln_gated"])
    assert_close(host(vox.adaln(dev(g["X"]), dev(g["shift"]), dev(g["scale"]), 1e-6)), g["adaln_modulate"])


def test_adaln_config3_bf16(vox, port):
    """x [8,2048,1024] bf16, shift/scale/gate [8,1024] ~N(0,0.1), residual ~N(0,1), eps 1e-6."""
    B, T, D = 8, 2048, 1024
    x = bf16r(port.normal((B, T, D), sid=60))
    res = bf16r(port.normal((B, T, D), sid=61))
    sh, sc, g = (bf16r(port.normal((B, D), 0.0, 0.1, sid=s)) for s in (62, 63, 64))
    want = bf16r(port.adaln(x, sh, sc, g, res))
    d = lambda a: dev(a, torch.bfloat16)  # noqa: E731
    out = vox.adaln(d(x), d(sh), d(sc), 1e-6, d(g), d(res))
    got = host(out)
    assert_close(got, want, BF16_TOL)
    # nearly every output is the oracle's bf16 value itself (statistics in f32 on the GPU, f64 on the CPU; the few
    # differences sit where residual and gate * m nearly cancel)
    assert np.mean(got.view(np.uint32) == want.view(np.uint32)) > 0.99
    assert_bitexact(host(vox.adaln(d(x), d(sh), d(sc), 1e-6, d(g), d(res))), got)


def test_adaln_f32_and_gated_add(vox, port):
    B, T, D = 3, 40, 256
    x = port.normal((B, T, D), sid=70)
    res = port.normal((B, T, D), sid=71)
    sh, sc, g = (port.normal((B, D), 0.0, 0.1, sid=s) for s in (72, 73, 74))
    assert_close(host(vox.adaln(dev(x), dev(sh), dev(sc), 1e-6, dev(g), dev(res))), port.adaln(x, sh, sc, g, res))
    assert_close(host(vox.adaln(dev(x), dev(sh), dev(sc), 1e-6)), port.adaln(x, sh, sc))
    h = dev(res)
    vox.gated_add(h, dev(g), dev(x))
    assert_close(host(h), port.gated_add(res, g, x))
    hb = dev(bf16r(res), torch.bfloat16)
    vox.gated_add(hb, dev(bf16r(g), torch.bfloat16), dev(bf16r(x), torch.bfloat16))
    assert_close(host(hb), bf16r(port.gated_add(bf16r(res), bf16r(g), bf16r(x))), BF16_TOL)


def test_bias_add(vox, port, golden):
    g = golden["bias"]
    assert_close(host(vox.bias_add(dev(g["y"]), dev(g["b"]))), g["out"])
    y = port.normal((333, 512), sid=80)
    b = port.normal((512,), sid=81)
    assert_close(host(vox.bias_add(dev(y), dev(b))), port.bias_add(y, b))
    yb = bf16r(y)
    assert_close(host(vox.bias_add(dev(yb, torch.bfloat16), dev(b))), bf16r(port.bias_add(yb, b)), BF16_TOL)


# ------------------------------------------------------------------ softmax

def test_softmax_golden(vox, golden):
    g = golden["softmax"]
    k = float(g["scale"])
    assert_close(host(vox.softmax_rows(dev(g["s"]), k, 64, 0)), g["causal"])
    assert_close(host(vox.softmax_rows(dev(g["s"]), k, 0, 0)), g["full"])
    assert_close(host(vox.softmax_rows(dev(g["s2"]), k, 16, 24)), g["causal_pos24"])


def test_softmax_config2(vox, port):
    """scores [16,1024,1024] ~N(0,3) x 1/sqrt(128), causal."""
    s = port.normal((16, 1024, 1024), 0.0, 3.0, sid=90)
    k = 1.0 / np.sqrt(128.0)
    want = port.softmax_rows(s, k, 1024, 0)
    out = vox.softmax_rows(dev(s), k, 1024, 0)
    got = host(out)
    assert_close(got, want)
    iq, ik = np.indices((1024, 1024))
    assert np.all(got[:, ik > iq] == 0.0)
    np.testing.assert_allclose(got.sum(-1, dtype=np.float64), 1.0, rtol=1e-5)
    # the full-read form with -inf above the diagonal gives the same rows
    sm = s.copy()
    sm[:, ik > iq] = -np.inf
    assert_close(host(vox.softmax_rows(dev(sm), k, 0, 0)), want)


@pytest.mark.parametrize("n", [1, 3, 64, 1000, 2048, 3000])
def test_softmax_lengths(vox, port, n):
    s = port.normal((2, 21, n), 0.0, 3.0, sid=n)
    assert_close(host(vox.softmax_rows(dev(s), 0.5, 21, 5)), port.softmax_rows(s, 0.5, 21, 5))
    assert_close(host(vox.softmax_rows(dev(s), 0.5, 0, 0)), port.softmax_rows(s, 0.5, 0, 0))
    assert_close(host(vox.softmax_rows(dev(s), -0.75, 21, 5)), port.softmax_rows(s, -0.75, 21, 5))  # unfolded scale
    xi = dev(s)
    vox.softmax_rows(xi, 0.5, 21, 5, out=xi)
    assert_close(host(xi), port.softmax_rows(s, 0.5, 21, 5))


# ------------------------------------------------------------------ activations

def test_activations_golden(vox, golden):
    g = golden["act"]
    assert_close(host(vox.silu_mul(dev(g["g"]), dev(g["u"]))), g["silu_mul"])
    assert_close(host(vox.gelu(dev(g["xg"])[None], vox.GELU_ERF))[0], g["gelu_erf"], floor=1.0)
    assert_close(host(vox.gelu(dev(g["xg"])[None], vox.GELU_TANH))[0], g["gelu_tanh"], floor=1.0)
    assert_close(host(vox.gelu(dev(g["xg"])[None], vox.GELU_ERF))[0], g["gelu_inplace"], floor=1.0)
    x, al = dev(g["xs"]), dev(g["alpha"])
    assert_close(host(vox.snake(x, al, vox.SNAKE_HIFT)), g["snake_hift_cm"])
    assert_close(host(vox.snake(x, al, vox.SNAKE_HIFT, channel_major=False)), g["snake_hift_tm"])
    assert_bitexact(host(vox.snake(x, al, vox.SNAKE_KOKORO)), g["snake_kokoro_cm"])
    assert_bitexact(host(vox.snake(x, al, vox.SNAKE_KOKORO, channel_major=False)), g["snake_kokoro_tm"])
    assert_close(host(vox.snake(x, al, vox.SNAKE_BETA, beta=dev(g["inv_b"]), channel_major=False)), g["snake_beta_tm"])


def test_swiglu_config1(vox, port):
    """BASELINE config 1b: silu(g) * u with g, u [512,3072] ~N(0,1); also the fused gate|up layout and bf16."""
    g = port.normal((512, 3072), sid=100)
    u = port.normal((512, 3072), sid=101)
    want = port.silu_mul(g, u)
    assert_close(host(vox.silu_mul(dev(g), dev(u))), want)
    gu = np.concatenate([g, u], axis=1)
    assert_close(host(vox.swiglu_fused(dev(gu))), want)
    assert_close(host(vox.swiglu_fused(dev(gu[:, 1:-1].copy()))), port.swiglu_fused(gu[:, 1:-1]))  # I odd: scalar path
    gb, ub = bf16r(g), bf16r(u)
    assert_close(host(vox.silu_mul(dev(gb, torch.bfloat16), dev(ub, torch.bfloat16))), bf16r(port.silu_mul(gb, ub)), BF16_TOL)
    gi = dev(g)
    vox.silu_mul(gi, dev(u), out=gi)
    assert_close(host(gi), want)
    assert_close(host(vox.silu_mul(unaligned(g), unaligned(u))), want)


@pytest.mark.parametrize("n", [1, 5, 4099, 1 << 20])
def test_sweep_elementwise(vox, port, n):
    a = port.normal((n,), sid=110)
    b = port.normal((n,), sid=111)
    assert_bitexact(host(vox.add(dev(a), dev(b))), port.add(a, b))
    assert_bitexact(host(vox.mul(dev(a), dev(b))), port.mul(a, b))
    assert_close(host(vox.gelu(dev(a)[None]))[0], port.gelu(a, 0), floor=1.0)
    assert_close(host(vox.gelu(dev(a)[None], vox.GELU_TANH))[0], port.gelu(a, 1), floor=1.0)
    ab, bb = bf16r(a), bf16r(b)
    assert_bitexact(host(vox.add(dev(ab, torch.bfloat16), dev(bb, torch.bfloat16))), bf16r(port.add(ab, bb)))
    assert_bitexact(host(vox.mul(dev(ab, torch.bfloat16), dev(bb, torch.bfloat16))), bf16r(port.mul(ab, bb)))
    assert_close(host(vox.gelu(dev(ab, torch.bfloat16)[None]))[0], bf16r(port.gelu(ab, 0)), BF16_TOL, floor=1.0)
    assert_bitexact(host(vox.add(unaligned(a), unaligned(b))), port.add(a, b))


def test_snake_config4(vox, port):
    """HiFT Snake on x [16,512,24000] f32 channel-major, alpha ~U(0.2,2) per channel."""
    x = port.normal((16, 512, 24000), sid=120)
    al = port.uniform_arr((512,), 0.2, 2.0, sid=121)
    out = host(vox.snake(dev(x), dev(al), vox.SNAKE_HIFT))
    rows = [0, 1, 511, 512, 4095, 8191]
    for r in rows:
        b, c = divmod(r, 512)
        want = port.snake(x[b, c], al[c:c + 1], 0, inner=24000)
        # |d| <= 1e-5 |y|, or 1e-6 |x| where x + s^2/alpha nearly cancels
        d = np.abs(out[b, c] - want)
        assert np.all(d <= np.maximum(1e-5 * np.abs(want), 1e-6 * np.abs(x[b, c])) + 1e-30)
    # Kokoro form is bit-exact with Vox's fast_sin at full size (sampled rows)
    outk = host(vox.snake(dev(x), dev(al), vox.SNAKE_KOKORO))
    for r in rows:
        b, c = divmod(r, 512)
        assert_bitexact(outk[b, c], port.snake(x[b, c], al[c:c + 1], 2, inner=24000))


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_snake_layouts(vox, port, kind):
    al = port.uniform_arr((12,), 0.2, 2.0, sid=130)
    ib = port.uniform_arr((12,), 0.5, 1.5, sid=131) if kind == 1 else None
    for shape, cm in (((3, 12, 50), True), ((3, 12, 7), True), ((77, 12), False)):
        x = port.normal(shape, sid=132)
        inner = shape[-1] if cm else 1
        want = port.snake(x, al, kind, ib, inner=inner)
        got = host(vox.snake(dev(x), dev(al), kind, None if ib is None else dev(ib), channel_major=cm))
        if kind == 2:
            assert_bitexact(got, want)
        else:
            assert np.all(np.abs(got - want) <= np.maximum(1e-5 * np.abs(want), 1e-6 * np.abs(x)) + 1e-30)


@pytest.mark.parametrize("C", [6144, 6148])
def test_snake_wide_channels(vox, port, C):
    """Up to 6144 channels the (alpha, coef) pairs are folded into a per-CTA shared table; wider channel counts index
    alpha per vector. Both sides of the limit, both layouts, HiFT (within f32 rounding) and Kokoro (bit-exact)."""
    al = port.uniform_arr((C,), 0.2, 2.0, sid=133)
    for shape, cm in (((2, C, 8), True), ((5, C), False)):
        x = port.normal(shape, sid=134)
        for kind in (0, 2):
            want = port.snake(x, al, kind, None, inner=shape[-1] if cm else 1)
            got = host(vox.snake(dev(x), dev(al), kind, channel_major=cm))
            if kind == 2:
                assert_bitexact(got, want)
            else:
                assert np.all(np.abs(got - want) <= np.maximum(1e-5 * np.abs(want), 1e-6 * np.abs(x)) + 1e-30)


def test_snake_load_params(vox, port):
    al = port.uniform_arr((12,), 0.2, 2.0, sid=130)
    a, b = vox.load_snake(dev(al), dev(al[::-1].copy()))
    pa, pb = port.load_snake(al, al[::-1].copy())
    assert_close(host(a)[None], pa[None])
    assert_close(host(b)[None], pb[None])


# ------------------------------------------------------------------ dequantisation

def test_dequant_golden_bitexact(vox, golden):
    g = golden["dequant"]
    q8, q4, s32 = dev(g["q8"]), dev(g["q4"]), dev(g["scale_f32"])
    s16 = dev(g["scale_f16_bits"].view(np.float16))
    assert_bitexact(host(vox.dequant_q8(q8, s32, torch.float32)), g["q8_out"])
    assert_bitexact(host(vox.dequant_q8(q8, s16, torch.float32)), g["q8_out"])
    assert_bitexact(host(vox.dequant_q4(q4, s32, torch.float32)), g["q4_out"])
    assert_bitexact(host(vox.dequant_q4(q4, s16, torch.float32)), g["q4_out"])
    assert_bitexact(host(vox.dequant_q8(q8, s16)), bf16r(g["q8_out"]))
    assert_bitexact(host(vox.dequant_q4(q4, s16)), bf16r(g["q4_out"]))
    assert_bitexact(host(vox.dequant_q8(dev(g["quant_q8"]), dev(g["quant_q8_scale"]), torch.float32)), g["quant_q8_out"])
    assert_bitexact(host(vox.dequant_q4(dev(g["quant_q4"]), dev(g["quant_q4_scale"]), torch.float32)), g["quant_q4_out"])


def test_dequant_config4_bitexact(vox, port):
    """[4096,4096] q8 (full int8 range) and q4, f16 scales ~U(0.001,0.05) -> bf16, bit-exact."""
    rows = cols = 4096
    q8 = port.fill_i8((rows, cols), -128, 127, sid=140)
    q4 = port.fill_u8((rows, cols // 2), sid=141)
    s16 = port.uniform_arr((rows, cols // 32), 0.001, 0.05, sid=142).astype(np.float16)
    s32 = port.f16_to_f32(s16.view(np.uint16))
    want8 = port.dequant_q8(q8, s32)
    want4 = port.dequant_q4(q4, s32)
    assert_bitexact(host(vox.dequant_q8(dev(q8), dev(s16))), bf16r(want8))
    assert_bitexact(host(vox.dequant_q4(dev(q4), dev(s16))), bf16r(want4))
    assert_bitexact(host(vox.dequant_q8(dev(q8), dev(s32), torch.float32)), want8)
    assert_bitexact(host(vox.dequant_q4(dev(q4), dev(s32), torch.float32)), want4)


def test_dequant_edge_scales_bitexact(vox, port):
    """f16 scales at the edges of the format: +-0, negative, subnormal, the largest finite, +-inf and NaN, next to
    ordinary ones; bit-exact against float(code) * scale (kernels.cpp:450, 459-460), NaN where it is NaN."""
    rows, cols = 7, 4096
    q8 = port.fill_i8((rows, cols), -128, 127, sid=143)
    q8[:, :32] = np.arange(-128, 128, 8, dtype=np.int16).astype(np.int8)  # zero and the extremes in block 0
    q4 = port.fill_u8((rows, cols // 2), sid=144)
    special = np.array([0.0, -0.0, -0.02, 6e-8, 3e-5, 65504.0, np.inf, -np.inf, np.nan, 0.001, 0.05], np.float16)
    s16 = port.uniform_arr((rows, cols // 32), 0.001, 0.05, sid=145).astype(np.float16)
    flat = s16.reshape(-1)
    flat[::3] = np.resize(special, flat[::3].shape)
    s32 = port.f16_to_f32(s16.view(np.uint16))
    for fn, q, want in ((vox.dequant_q8, q8, port.dequant_q8(q8, s32)), (vox.dequant_q4, q4, port.dequant_q4(q4, s32))):
        for out_dt, ref in ((torch.float32, want), (torch.bfloat16, bf16r(want))):
            got = host(fn(dev(q), dev(s16), out_dt))
            nan = np.isnan(ref)
            np.testing.assert_array_equal(np.isnan(got), nan)
            assert_bitexact(np.where(nan, 0, got), np.where(nan, 0, ref))


def test_dequant_small_shapes(vox, port):
    for rows, cols in ((1, 32), (3, 64), (5, 96), (0, 32)):
        q8 = port.fill_i8((rows, cols), -128, 127, sid=150)
        q4 = port.fill_u8((rows, cols // 2), sid=151)
        s = port.uniform_arr((rows, cols // 32), 0.001, 0.05, sid=152)
        if rows:
            assert_bitexact(host(vox.dequant_q8(dev(q8), dev(s), torch.float32)), port.dequant_q8(q8, s))
            assert_bitexact(host(vox.dequant_q4(dev(q4), dev(s), torch.float32)), port.dequant_q4(q4, s))
        else:
            assert vox.dequant_q8(dev(q8), dev(s)).numel() == 0
    with pytest.raises(vox.VoxCudaError):
        vox.dequant_q8(dev(np.zeros((2, 48), np.int8)), dev(np.ones((2, 1), np.float32)))


# ------------------------------------------------------------------ reductions

@pytest.mark.parametrize("n", [1, 4, 33, 4096, 4100])
def test_row_reduce_bitexact_order(vox, port, n):
    x = port.normal((129, n), sid=160 + n)
    for op in (0, 1, 2):
        got = host(vox.row_reduce(dev(x), op))
        assert_bitexact(got, port.row_reduce(x, op, W=4))
        assert_bitexact(host(vox.row_reduce(unaligned(x), op)), got)  # scalar path, same order
        f64 = port.row_reduce_f64(x, op)
        scale = np.abs(x).sum(-1) if op == 0 else np.abs(f64)
        assert np.all(np.abs(got - f64) <= 1e-5 * scale + 1e-30)
    xb = bf16r(x)
    for op in (0, 1, 2):
        assert_bitexact(host(vox.row_reduce(dev(xb, torch.bfloat16), op)), port.row_reduce(xb, op, W=8))


def test_global_sum_deterministic_across_shard_counts(vox, port):
    from vox_b200.shard import shard_rows

    R, n = 3000, 4096
    x = port.normal((R, n), sid=170)
    xd = dev(x)
    slots1 = host(vox.global_sum_partials(xd, 0, R))
    np.testing.assert_array_equal(slots1, port.global_sum_slots(port.row_reduce(x, 0), 0, R))
    whole = host(vox.global_sum_finish(dev(slots1)))[0]
    assert whole == port.global_sum_finish(slots1)
    assert abs(whole - float(np.sum(x, dtype=np.float64))) <= 1e-6 * float(np.abs(x).sum())
    for world in (2, 4, 8, 3, 5, 6, 7):
        acc = torch.zeros(840, dtype=torch.float64, device="cuda")
        for k in range(world):
            r0, rows = shard_rows(R, world, k)
            acc += vox.global_sum_partials(xd[r0:r0 + rows], r0, R)
        assert host(vox.global_sum_finish(acc))[0] == whole
    with pytest.raises(vox.VoxCudaError):
        vox.global_sum_partials(xd[1:10], 1, R)


def test_cpu_tensor_is_rejected(vox):
    with pytest.raises(vox.VoxCudaError):
        vox.add(torch.ones(4), torch.ones(4))
    with pytest.raises(vox.VoxCudaError):
        vox.add(torch.ones(4, dtype=torch.float64, device="cuda"), torch.ones(4, dtype=torch.float64, device="cuda"))


def test_no_device_side_timeouts(vox):
    """Every bounded wait of the row pipeline completed during the tests above (flag read and cleared)."""
    import ctypes

    flags = ctypes.c_uint(7)
    vox._check(vox.lib.vox_cuda_device_error(ctypes.byref(flags)))
    assert flags.value == 0
