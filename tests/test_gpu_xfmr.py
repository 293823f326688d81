"""GPU parity tests of the transformer elementwise chain (vox_cuda_rope_table, vox_cuda_qkv_rope,
vox_cuda_add_rmsnorm) through the C ABI, against the oracle's restatement of transformer_forward's per-token steps
(kernels.cpp:793-833, pinned to the reference's own rmsnorm / rope_apply by tests/golden/xfmr.npz).

Bars: the RoPE rotation and the K/V cache writes are bit-exact given the same cos/sin table (the rotation rounds
every product separately, as the CPU); the device table is within 2 ulp of libm's cosf/sinf; head norms and the
RMSNorm after the residual update are within 1e-5 of the row scale (their sum of squares is a warp tree, not the
CPU's sequential sum); the residual update itself is bit-exact (f32) or the bf16 rounding of the f32 result.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from test_gpu_parity import BF16_TOL, assert_bitexact, assert_close, bf16r, dev, host

pytestmark = pytest.mark.gpu


def _chain_inputs(port, m, heads, kv, hd, pos0, sid=60, norms=True):
    qkv = port.normal((m, (heads + 2 * kv) * hd), sid=sid)
    qn = port.normal((hd,), 1.0, 0.1, sid=sid + 1) if norms else None
    kn = port.normal((hd,), 1.0, 0.1, sid=sid + 2) if norms else None
    inv = port.rope_inv_freq(hd, 1e6)
    cs = port.rope_table(inv, pos0, m)
    return qkv, qn, kn, inv, cs


def _run_gpu(vox, qkv, qn, kn, cs, heads, kv, hd, pos0, rows, ring=0, sentinel=None, misalign=False):
    kd = kv * hd
    kc = dev(sentinel[0]) if sentinel is not None else torch.zeros((rows, kd), device="cuda")
    vc = dev(sentinel[1]) if sentinel is not None else torch.zeros((rows, kd), device="cuda")
    if misalign:  # one float past a 16-byte boundary: the general kernel
        buf = torch.empty(qkv.size + 1, device="cuda")
        x = buf[1:].view(qkv.shape)
        x.copy_(dev(qkv))
        assert x.data_ptr() % 16 != 0
    else:
        x = dev(qkv)
    q = vox.qkv_rope(x, dev(cs), heads, kv, hd, kc, vc, pos0, q_norm_w=None if qn is None else dev(qn),
                     k_norm_w=None if kn is None else dev(kn), ring=ring)
    return host(q), host(kc), host(vc)


def test_rope_table_within_2ulp_of_libm(vox, port):
    for hd, theta in ((128, 1e6), (64, 1e4)):
        inv = vox.rope_inv_freq(hd, theta)
        assert_bitexact(host(inv), port.rope_inv_freq(hd, theta))  # the model-load constant of kernels.cpp:734-738
        for pos0, m in ((0, 4096), (100000, 64)):
            got = host(vox.rope_table(inv, pos0, m))
            want = port.rope_table(port.rope_inv_freq(hd, theta), pos0, m)
            assert np.abs(got.astype(np.float64) - want).max() <= 2.4e-7


def test_qkv_rope_golden(vox, golden):
    g = golden["xfmr"]
    heads, kv, hd, m, pos0 = (int(v) for v in g["dims"])
    from oracle.oracle import port as _port

    cs = _port().rope_table(g["inv_freq"], pos0, m)
    q, kc, vc = _run_gpu(vox, g["qkv"], None, None, cs, heads, kv, hd, pos0, pos0 + m)
    assert_bitexact(q, g["q_rope"])
    assert_bitexact(kc[pos0:], g["k_rope"])
    assert_bitexact(vc[pos0:], g["qkv"][:, (heads + kv) * hd:])
    q, kc, vc = _run_gpu(vox, g["qkv"], g["qn"], g["kn"], cs, heads, kv, hd, pos0, pos0 + m)
    assert_close(q, g["q_norm_rope"])
    assert_close(kc[pos0:], g["k_norm_rope"])


@pytest.mark.parametrize("hd,misalign", [(64, False), (128, False), (256, False), (128, True), (96, False), (32, False)])
def test_qkv_rope_head_dims_and_paths(vox, port, hd, misalign):
    heads, kv, m, pos0 = 8, 2, 19, 300
    qkv, qn, kn, inv, cs = _chain_inputs(port, m, heads, kv, hd, pos0, norms=False)
    rows = pos0 + m + 3
    sent = (port.normal((rows, kv * hd), sid=70), port.normal((rows, kv * hd), sid=71))
    q, kc, vc = _run_gpu(vox, qkv, None, None, cs, heads, kv, hd, pos0, rows, sentinel=sent, misalign=misalign)
    wq, wk, wv = port.qkv_rope(qkv, None, None, cs, heads, kv, hd, pos0, kc=sent[0], vc=sent[1])
    assert_bitexact(q, wq)
    assert_bitexact(kc, wk)  # includes the rows outside pos0 .. pos0+m-1, which stay as they were
    assert_bitexact(vc, wv)
    qn = port.normal((hd,), 1.0, 0.1, sid=72)
    kn = port.normal((hd,), 1.0, 0.1, sid=73)
    q, kc, vc = _run_gpu(vox, qkv, qn, kn, cs, heads, kv, hd, pos0, rows, sentinel=sent, misalign=misalign)
    wq, wk, wv = port.qkv_rope(qkv, qn, kn, cs, heads, kv, hd, pos0, kc=sent[0], vc=sent[1])
    assert_close(q, wq)
    assert_close(kc[pos0:pos0 + m], wk[pos0:pos0 + m])
    assert_bitexact(kc[:pos0], wk[:pos0])
    assert_bitexact(vc, wv)


def test_qkv_rope_ring_slots(vox, port):
    heads, kv, hd, m, pos0, ring = 4, 4, 128, 8, 45, 8  # positions 45 .. 52 wrap from slot 7 to slot 0
    qkv, qn, kn, inv, cs = _chain_inputs(port, m, heads, kv, hd, pos0)
    sent = (port.normal((ring, kv * hd), sid=74), port.normal((ring, kv * hd), sid=75))
    q, kc, vc = _run_gpu(vox, qkv, qn, kn, cs, heads, kv, hd, pos0, ring, ring=ring, sentinel=sent)
    wq, wk, wv = port.qkv_rope(qkv, qn, kn, cs, heads, kv, hd, pos0, kc=sent[0], vc=sent[1], ring=ring)
    assert_close(q, wq)
    assert_close(kc, wk)
    assert_bitexact(vc, wv)
    with pytest.raises(vox.VoxCudaError) as e:  # more tokens than slots: rejected, not raced
        _run_gpu(vox, port.normal((ring + 1, (heads + 2 * kv) * hd), sid=76), qn, kn, port.rope_table(inv, pos0, ring + 1),
                 heads, kv, hd, pos0, ring, ring=ring, sentinel=sent)
    assert e.value.status == -6


def test_qkv_rope_decode_and_prefill_sizes(vox, port):
    """Decode (one token, GQA 32/8) and a Qwen3-0.6B-shaped prefill chunk (16/8 heads of 128, 8192 tokens)."""
    for m, heads, kv, pos0 in ((1, 32, 8, 4095), (8192, 16, 8, 0)):
        hd = 128
        qkv, qn, kn, inv, cs_host = _chain_inputs(port, m, heads, kv, hd, pos0, sid=80)
        # the device table feeds the kernel here (as in the product): compare with the oracle on the same table
        cs = host(vox.rope_table(dev(inv), pos0, m))
        q, kc, vc = _run_gpu(vox, qkv, qn, kn, cs, heads, kv, hd, pos0, pos0 + m)
        wq, wk, wv = port.qkv_rope(qkv, qn, kn, cs, heads, kv, hd, pos0)
        assert_close(q, wq)
        assert_close(kc[pos0:], wk[pos0:])
        assert_bitexact(vc[pos0:], wv[pos0:])


def test_qkv_rope_rejects_odd_head_dim(vox):
    x = torch.zeros((1, 3 * 7), device="cuda")
    kc = torch.zeros((1, 7), device="cuda")
    with pytest.raises(vox.VoxCudaError) as e:
        vox.qkv_rope(x, torch.zeros((1, 3, 2), device="cuda"), 1, 1, 7, kc, kc.clone(), 0)
    assert e.value.status == -6


def test_add_rmsnorm_golden(vox, golden):
    g = golden["xfmr"]
    for ls, hw, xw in ((g["ls"], g["h_ls"], g["xn_ls"]), (None, g["h_no"], g["xn_no"])):
        h = dev(g["h"])
        xn = vox.add_rmsnorm(h, dev(g["d"]), dev(g["w"]), 1e-6, layer_scale=None if ls is None else dev(ls))
        assert_bitexact(host(h), hw)
        assert_close(host(xn), xw)


@pytest.mark.parametrize("n", [1024, 1000, 33, 8192])
def test_add_rmsnorm_f32(vox, port, n):
    rows = 257
    h0, d = port.normal((rows, n), sid=90), port.normal((rows, n), sid=91)
    w, ls = port.normal((n,), 1.0, 0.02, sid=92), port.normal((n,), 0.0, 0.1, sid=93)
    for lsv in (ls, None):
        h = dev(h0)
        xn = vox.add_rmsnorm(h, dev(d), dev(w), 1e-6, layer_scale=None if lsv is None else dev(lsv))
        wh, wx = port.add_rmsnorm(h0, d, lsv, w)
        assert_bitexact(host(h), wh)
        assert_close(host(xn), wx)


@pytest.mark.parametrize("n", [1024, 4096, 40])
def test_add_rmsnorm_bf16(vox, port, n):
    rows = 129
    h0, d = bf16r(port.normal((rows, n), sid=94)), bf16r(port.normal((rows, n), sid=95))
    w, ls = port.normal((n,), 1.0, 0.02, sid=96), port.normal((n,), 0.0, 0.1, sid=97)
    h = dev(h0, torch.bfloat16)
    xn = vox.add_rmsnorm(h, dev(d, torch.bfloat16), dev(w), 1e-6, layer_scale=dev(ls))
    wh, wx = port.add_rmsnorm(h0, d, ls, w)
    assert_bitexact(host(h), bf16r(wh))  # the f32 sum, rounded once to bf16
    assert_close(host(xn), wx, tol=BF16_TOL)
