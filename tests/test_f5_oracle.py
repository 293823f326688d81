"""CPU tests of the F5 DiT oracle (oracle/f5.py) and of the vox_cuda_f5 argument checks.

The oracle's pieces are checked against the reference's own outputs (tests/golden, written by the reference compiled
from its sources): the modulated LayerNorm (adaLN without gate, f5.cpp:617-632), GELU-tanh (f5.cpp:93-96) and the
scaled row softmax (kernels.cpp:725-732, the softmax of f5.cpp:651-661). The argument checks of vox_cuda_f5_create run
before any device work, so they need no GPU.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import f5 as F5


def test_modulate_matches_reference(golden):
    g = golden["norm"]
    for b in range(g["X"].shape[0]):
        want = g["adaln_modulate"][b].astype(np.float64)
        got = F5.modulate(g["X"][b].astype(np.float64), g["scale"][b].astype(np.float64), g["shift"][b].astype(np.float64))
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())


def test_gelu_tanh_matches_reference(golden):
    g = golden["act"]
    x = g["xg"].astype(np.float64)
    assert np.all(np.abs(F5.gelu_tanh(x) - g["gelu_tanh"]) <= 2e-7 * np.abs(x) + 1e-7)


def test_softmax_matches_reference(golden):
    g = golden["softmax"]
    assert np.abs(F5.softmax(g["s"], float(g["scale"])) - g["full"]).max() <= 1e-6


def test_rope_table_is_the_float32_construction():
    c, s = F5.rope_table(300, 64)
    assert c.dtype == np.float32 and c.shape == (300, 32)
    inv = np.float32(1.0 / 10000.0 ** (2 * 5 / 64))
    a = np.float32(np.float32(299) * inv)
    assert c[299, 5] == np.float32(np.cos(np.float64(a))) and s[299, 5] == np.float32(np.sin(np.float64(a)))
    assert np.all(c[0] == 1.0) and np.all(s[0] == 0.0)


def test_conv1d_matches_a_direct_sum():
    rng = np.random.default_rng(3)
    T, cin, groups, K = 9, 8, 2, 5
    x, w, b = rng.standard_normal((T, cin)), rng.standard_normal((6, cin // groups, K)), rng.standard_normal(6)
    y = F5.conv1d(x, w, b, groups)
    for t in range(T):
        for o in range(6):
            g = o // 3
            acc = b[o] + sum(w[o, i, k] * x[t + k - K // 2, g * 4 + i] for i in range(4) for k in range(K) if 0 <= t + k - K // 2 < T)
            assert abs(y[t, o] - acc) < 1e-12


def test_dit_of_zero_blocks_is_the_output_head():
    rng = np.random.default_rng(0)
    R, D, O = 6, 16, 5
    h, ts = rng.standard_normal((R, D)), rng.standard_normal(D)
    norm_out, proj_out = rng.standard_normal((2 * D, D)) * 0.1, rng.standard_normal((O, D))
    out, h2 = F5.dit(h, ts, [], norm_out, proj_out, heads=2, dim_head=8, batch=2, frames=3)
    fin = norm_out @ ts
    np.testing.assert_allclose(out, F5.modulate(h, fin[:D], fin[D:]) @ proj_out.T, rtol=1e-12)
    np.testing.assert_array_equal(h2, h)


from vox_b200 import _F5Block as _Block, _F5Desc as _Desc  # the C layouts of vox_cuda_f5_block_weights / vox_cuda_f5_desc


@pytest.mark.parametrize("field,value", [("dim_head", 15), ("pe_attn_head", 5), ("math", 7), ("depth", 0), ("frames", 0),
                                         ("in_proj", 8)])
def test_f5_create_rejects_bad_descriptions(vox_lib, field, value):
    L = vox_lib.lib
    blk = (_Block * 1)(_Block(*([8] * 7)))
    d = _Desc(64, 4, 16, 2, 1, 0, 20, 2, 10, 0, blk, 8, 8, None, None, 0)
    setattr(d, field, value)
    h = ctypes.c_void_p()
    assert L.vox_cuda_f5_create(ctypes.byref(d), None, ctypes.byref(h)) == -6
    assert h.value is None
    assert L.vox_cuda_last_error()


def test_f5_create_rejects_null_weights(vox_lib):
    L = vox_lib.lib
    blk = (_Block * 1)(_Block(8, 8, 8, None, 8, 8, 8))
    d = _Desc(64, 4, 16, 2, 1, 0, 20, 2, 10, 0, blk, 8, 8, None, None, 0)
    h = ctypes.c_void_p()
    assert L.vox_cuda_f5_create(ctypes.byref(d), None, ctypes.byref(h)) == -6
    assert L.vox_cuda_f5_create(None, None, ctypes.byref(h)) == -6
    L.vox_cuda_f5_destroy(None)


def f5_golden_model(g):
    """The golden F5 model (tests/golden/f5.npz, written by make_golden.py from the reference): the residual stream
    entering the blocks (the oracle's input embedding of [x, cond, temb]), ts, and the weights."""
    keys = ("dim", "depth", "heads", "dim_head", "ff_mult", "text_dim", "text_rows", "mel_dim", "pe_attn_head")
    dims = dict(zip(keys, (int(v) for v in g["dims"])))
    B, N, M = g["x"].shape
    h = F5.embed(g["x"], g["cond"], g["temb"], g["in_proj"], g["in_proj_b"], g["pos1_w"], g["pos1_b"], g["pos2_w"], g["pos2_b"])
    blocks = [{k: g[f"b{l}_{k}"] for k in ("ada", "q", "k", "v", "o", "ff1", "ff2", "ada_b", "q_b", "k_b", "v_b", "o_b", "ff1_b",
                                           "ff2_b")} for l in range(dims["depth"])]
    return dims, B, N, h, blocks


def test_dit_matches_reference_dit_forward(golden):
    """The oracle's input embedding and DiT equal F5Model::dit_forward of the reference (f32 CPU arithmetic against
    float64: within 1e-5 of the output's RMS)."""
    g = golden["f5"]
    dims, B, N, h, blocks = f5_golden_model(g)
    out, _ = F5.dit(h, g["ts"], blocks, g["norm_out"], g["proj_out"], heads=dims["heads"], dim_head=dims["dim_head"], batch=B,
                    frames=N, pe_attn_head=dims["pe_attn_head"], norm_out_b=g["norm_out_b"], proj_out_b=g["proj_out_b"])
    want = g["out"].reshape(B * N, -1).astype(np.float64)
    err = np.abs(out - want).max() / np.sqrt(np.mean(want ** 2))
    assert err <= 1e-5, err
