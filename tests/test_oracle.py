"""CPU tests of the parity oracle: the C restatement of Vox's arithmetic against the reference's own known-answer
vectors and against the golden fixtures recorded from the reference's compiled CPU code (tests/golden/)."""

from __future__ import annotations

import numpy as np
import pytest


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def assert_bitexact(a, b):
    np.testing.assert_array_equal(bits(np.asarray(a, np.float32)), bits(np.asarray(b, np.float32)))


# Random123 known-answer vectors for Philox4x32-10, as checked by the reference (tests/test_core.cpp:35-43).
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0), (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", PHILOX_KAT)
def test_philox_kat(port, ctr, key, want):
    assert tuple(int(v) for v in port.philox_block(ctr, key)) == want


def test_uniform_and_noise_match_reference(port, golden):
    g = golden["gen"]
    for si, seed in enumerate(g["uniform_seeds"]):
        for d in (0, 1):
            got = np.array([port.uniform(int(seed), f, 7, d) for f in range(256)], np.float32)
            assert_bitexact(got, g["uniform"][si, d])
    assert_bitexact(port.f5_noise(0, 0, 1001), g["noise_0_0"])
    assert_bitexact(port.f5_noise(12345, 3, 513), g["noise_12345_3"])


def test_uniform_range_and_determinism(port):
    u = port.fill(4096, 0, 0.0, 1.0, seed=7, sid=3)
    assert u.min() >= 0.0 and u.max() < 1.0
    assert_bitexact(u, port.fill(4096, 0, 0.0, 1.0, seed=7, sid=3))
    assert not np.array_equal(u, port.fill(4096, 0, 0.0, 1.0, seed=8, sid=3))
    # a shard drawn with a counter offset equals the slice of the whole
    assert_bitexact(port.fill(100, 1, 0.0, 1.0, seed=7, c0=1000), port.fill(1100, 1, 0.0, 1.0, seed=7)[1000:])


def test_norms_golden(port, golden):
    g = golden["norm"]
    assert_bitexact(port.rmsnorm(g["x"], g["w"], 1e-6), g["rmsnorm"])
    assert_bitexact(port.rmsnorm(g["x33"], g["w"][:33], 1e-6), g["rmsnorm33"])
    assert_bitexact(port.layernorm(g["x"], g["w"], g["b"], 1e-5), g["layernorm"])
    assert_bitexact(port.layernorm(g["x"], g["w"], None, 1e-5), g["layernorm_nob"])
    assert_bitexact(port.layernorm(g["x"], g["w"], g["b"], 1e-6, modulate=True), g["ln_modulate"])
    assert_bitexact(port.layernorm(g["x"], None, None, 1e-6), g["ln_plain"])
    assert_bitexact(port.adaln(g["X"], g["shift"], g["scale"], g["gate"], g["res"]), g["adaln_gated"])
    assert_bitexact(port.adaln(g["X"], g["shift"], g["scale"]), g["adaln_modulate"])


def test_softmax_golden(port, golden):
    g = golden["softmax"]
    k = float(g["scale"])
    assert_bitexact(port.softmax_rows(g["s"], k, 64, 0), g["causal"])
    assert_bitexact(port.softmax_rows(g["s"], k, 0, 0), g["full"])
    assert_bitexact(port.softmax_rows(g["s2"], k, 16, 24), g["causal_pos24"])
    # Vox's AVX2 exp polynomial variant (nn::softmax_fast) agrees to a few ulp
    np.testing.assert_allclose(port.softmax_rows(g["s"], k, 64, 0), g["causal_fast"], rtol=2e-6, atol=1e-7)
    # the causal rows are exactly zero past the diagonal and sum to 1
    c = g["causal"]
    iq, ik = np.indices(c.shape[1:])
    assert np.all(c[:, ik > iq] == 0)
    np.testing.assert_allclose(c.sum(-1), 1.0, rtol=1e-6)


def test_activations_golden(port, golden):
    g = golden["act"]
    assert_bitexact(port.silu_mul(g["g"], g["u"]), g["silu_mul"])
    assert_bitexact(port.gelu(g["xg"], 0), g["gelu_erf"])
    assert_bitexact(port.gelu(g["xg"], 1), g["gelu_tanh"])
    np.testing.assert_allclose(port.gelu(g["xg"], 0), g["gelu_inplace"], rtol=1e-6, atol=3e-7)
    assert_bitexact(port.snake(g["xs"], g["alpha"], 0, inner=100), g["snake_hift_cm"])
    assert_bitexact(port.snake(g["xs"], g["alpha"], 0, inner=1), g["snake_hift_tm"])
    assert_bitexact(port.snake(g["xs"], g["alpha"], 2, inner=100), g["snake_kokoro_cm"])
    assert_bitexact(port.snake(g["xs"], g["alpha"], 2, inner=1), g["snake_kokoro_tm"])
    assert_bitexact(port.snake(g["xs"], g["alpha"], 1, g["inv_b"], inner=1), g["snake_beta_tm"])
    assert_bitexact(np.array([port.fast_sin(v) for v in g["fast_sin_x"]], np.float32), g["fast_sin"])


def test_dequant_golden(port, golden):
    g = golden["dequant"]
    assert_bitexact(port.f16_to_f32(g["scale_f16_bits"]), g["scale_f32"])
    assert_bitexact(port.dequant_q8(g["q8"], g["scale_f32"]), g["q8_out"])
    assert_bitexact(port.dequant_q4(g["q4"], g["scale_f32"]), g["q4_out"])
    assert_bitexact(port.dequant_q8(g["quant_q8"], g["quant_q8_scale"]), g["quant_q8_out"])
    assert_bitexact(port.dequant_q4(g["quant_q4"], g["quant_q4_scale"]), g["quant_q4_out"])
    assert g["q8"].min() == -128 and g["q8"].max() == 127  # full int8 range, including -128
    # Q4 round trip of the reference quantizer: error at most two steps (tests/test_core.cpp:477-485)
    step = np.repeat(np.abs(g["quant_q4_scale"]), 32, axis=1)
    assert np.all(np.abs(g["quant_q4_out"] - g["wq"]) <= step * 2.001)


def test_bias_golden(port, golden):
    g = golden["bias"]
    assert_bitexact(port.bias_add(g["y"], g["b"]), g["out"])


def test_bf16_rounding(port):
    x = np.array([1.0, 1.00390625, 1.005859375, -3.1415927, 65504.0, 1e-30, 0.0, -0.0], np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    want = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # python/vox/build.py:94-97
    np.testing.assert_array_equal(port.bf16_round(x), want)


def test_row_reduce_order_vs_f64(port):
    x = port.normal((37, 4096), sid=50)
    for op in (0, 1, 2):
        a = port.row_reduce(x, op).astype(np.float64)
        b = port.row_reduce_f64(x, op)
        scale = np.abs(x).sum(-1) if op != 1 else np.abs(b)
        if op == 2:
            scale = b
        assert np.all(np.abs(a - b) <= 1e-5 * scale + 1e-30)
    # the documented order is independent of the row count
    np.testing.assert_array_equal(port.row_reduce(x[:5], 0), port.row_reduce(x, 0)[:5])


def test_global_sum_order_independent_of_shards(port):
    from vox_b200.shard import shard_rows

    R, n = 1000, 64
    x = port.normal((R, n), sid=51)
    rowsum = port.row_reduce(x, 0)
    whole = port.global_sum_finish(port.global_sum_slots(rowsum, 0, R))
    for world in (2, 3, 4, 5, 6, 7, 8):
        acc = np.zeros(840)
        for k in range(world):
            r0, rows = shard_rows(R, world, k)
            acc += port.global_sum_slots(rowsum[r0:r0 + rows], r0, R)
        assert port.global_sum_finish(acc) == whole
    assert abs(whole - float(np.sum(x, dtype=np.float64))) <= 1e-6 * float(np.abs(x).sum())


def test_xfmr_chain_golden(port, golden):
    """The split + head norm + RoPE + cache write and the residual update + RMSNorm restatements reproduce the
    reference's rmsnorm / rope_apply / rope_inv_freq outputs bit for bit (the table from libm's cosf/sinf, as
    rope_apply computes it)."""
    g = golden["xfmr"]
    heads, kv, hd, m, pos0 = (int(v) for v in g["dims"])
    assert_bitexact(port.rope_inv_freq(hd, 1e6), g["inv_freq"])
    assert_bitexact(port.rope_inv_freq(64, 1e4), g["inv_freq_64"])
    cs = port.rope_table(g["inv_freq"], pos0, m)
    for qn, kn, qw, kw in ((g["qn"], g["kn"], g["q_norm_rope"], g["k_norm_rope"]), (None, None, g["q_rope"], g["k_rope"])):
        q, kc, vc = port.qkv_rope(g["qkv"], qn, kn, cs, heads, kv, hd, pos0)
        assert_bitexact(q, qw)
        assert_bitexact(kc[pos0:], kw)
        assert_bitexact(vc[pos0:], g["qkv"][:, (heads + kv) * hd:])
        assert not kc[:pos0].any() and not vc[:pos0].any()  # rows before pos0 untouched
    # ring slots: token i lands in row (pos0 + i) % ring
    q, kc, vc = port.qkv_rope(g["qkv"], None, None, cs, heads, kv, hd, pos0, ring=3)
    for i in range(m):
        if i >= m - 3:
            assert_bitexact(kc[(pos0 + i) % 3], g["k_rope"][i])
    for ls, hw, xw in ((g["ls"], g["h_ls"], g["xn_ls"]), (None, g["h_no"], g["xn_no"])):
        h, xn = port.add_rmsnorm(g["h"], g["d"], ls, g["w"])
        assert_bitexact(h, hw)
        assert_bitexact(xn, xw)


def test_gemv_golden(port, golden):
    """The float-activation GEMV restatement (accumulated in double) agrees with the reference's f32 matmul to within
    f32 rounding of the dot products: |d| <= 1e-6 * sum_k |w x|."""
    g = golden["gemv"]
    for key, q4, m, bias in (("q8_m9", False, 9, True), ("q8_m3", False, 3, True), ("q4_m3", True, 3, True),
                             ("q4_m1_nobias", True, 1, False)):
        y, bound = port.gemv(g["q4" if q4 else "q8"], g["scale"], g["x"][:m], g["bias"] if bias else None, q4=q4)
        assert np.all(np.abs(y.astype(np.float64) - g[key]) <= 1e-6 * bound + 1e-7), key


def test_reference_library_matches_golden(golden):
    from oracle.oracle import ref

    R = ref()
    if R is None:
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not present on this machine")
    g = golden["norm"]
    assert_bitexact(R.rmsnorm(g["x"], g["w"], 1e-6), g["rmsnorm"])
    s = golden["softmax"]
    assert_bitexact(R.softmax_rows(s["s"], float(s["scale"]), 64, 0), s["causal"])
    d = golden["dequant"]
    assert_bitexact(R.mat_rows(d["q8"], d["scale_f32"]), d["q8_out"])
    x = golden["xfmr"]
    heads, kv, hd, m, pos0 = (int(v) for v in x["dims"])
    q, k = R.qk_norm_rope(x["qkv"][:, :heads * hd], x["qkv"][:, heads * hd:(heads + kv) * hd], x["qn"], x["kn"], x["inv_freq"],
                          heads, kv, hd, pos0)
    assert_bitexact(q, x["q_norm_rope"])
    assert_bitexact(k, x["k_norm_rope"])
