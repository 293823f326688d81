"""GPU parity tests of the F5 DiT step (vox_cuda_f5_*, one CUDA graph): against the reference's own F5Model::dit_forward
(tests/golden/f5.npz, a tiny model run by the reference) and against the numpy restatement of it (oracle/f5.py, pinned to
the same golden), with a bias on every linear as F5 checkpoints carry.

Bars, relative to the RMS of the oracle's output: f32 GEMMs 2e-5 (the sums' order and the f32 LayerNorm statistics
differ from the f64 oracle); tensor cores with TF32 inputs 2e-2, with bf16 inputs 8e-2 (input rounding of 2^-11 and
2^-8 through two blocks; the bf16 mode with dim_head 64 also rounds the attention probabilities and every GEMM input
to bf16). Replays of the captured graph are bit-identical and read the inputs afresh.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import f5 as F5

pytestmark = pytest.mark.gpu


def _model(seed, D, H, HD, FF, depth, out_dim):
    """Random weights and biases (every linear biased, as F5 checkpoints are)."""
    rng = np.random.default_rng(seed)
    inner = H * HD
    mk = lambda o, i, s=1.0: (rng.standard_normal((o, i)) * s / np.sqrt(i)).astype(np.float32)  # noqa: E731
    bias = lambda o: (rng.standard_normal(o) * 0.1).astype(np.float32)  # noqa: E731
    blocks = []
    for _ in range(depth):
        b = {"ada": mk(6 * D, D, 0.3), "q": mk(inner, D), "k": mk(inner, D), "v": mk(inner, D), "o": mk(D, inner), "ff1": mk(FF, D),
             "ff2": mk(D, FF)}
        b.update({k + "_b": bias(b[k].shape[0]) for k in list(b)})
        blocks.append(b)
    return blocks, mk(2 * D, D, 0.3), mk(out_dim, D), bias(2 * D), bias(out_dim)


def _dev(blocks, norm_out, proj_out, norm_out_b=None, proj_out_b=None):
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    return [{k: t(v) for k, v in b.items()} for b in blocks], t(norm_out), t(proj_out), t(norm_out_b), t(proj_out_b)


def _plan(vox, dev_model, **kw):
    blocks, norm_out, proj_out, nb, pb = dev_model
    return vox.F5Dit(blocks, norm_out, proj_out, norm_out_b=nb, proj_out_b=pb, **kw)


def _oracle(model, h, ts, **kw):
    blocks, norm_out, proj_out, nb, pb = model
    return F5.dit(h, ts, blocks, norm_out, proj_out, norm_out_b=nb, proj_out_b=pb, **kw)


@pytest.mark.parametrize("math,bar", [("f32", 2e-5), ("tf32", 2e-2)])
def test_f5_step_matches_reference_dit_forward(vox, golden, math, bar):
    """The golden F5 model (tests/golden/f5.npz): the step from the residual stream after the input embedding equals
    the reference's F5Model::dit_forward output (every linear biased, RoPE on the first head only)."""
    from test_f5_oracle import f5_golden_model

    g = golden["f5"]
    dims, B, N, h, blocks = f5_golden_model(g)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()  # noqa: E731
    plan = vox.F5Dit([{k: t(v) for k, v in b.items()} for b in blocks], t(g["norm_out"]), t(g["proj_out"]), heads=dims["heads"],
                     dim_head=dims["dim_head"], batch=B, frames=N, pe_attn_head=dims["pe_attn_head"], math=math,
                     norm_out_b=t(g["norm_out_b"]), proj_out_b=t(g["proj_out_b"]))
    out = plan.step(t(h), t(g["ts"])).cpu().numpy()
    plan.close()
    want = g["out"].reshape(B * N, -1).astype(np.float64)
    assert _rel(out, want) <= bar, _rel(out, want)


def _rel(got, want):
    return np.abs(np.asarray(got, np.float64) - want).max() / np.sqrt(np.mean(want ** 2))


CFG = dict(D=64, H=4, HD=16, FF=128, depth=2, out_dim=20)


@pytest.mark.parametrize("pe_attn_head", [0, 2])
@pytest.mark.parametrize("math,bar", [("f32", 2e-5), ("tf32", 2e-2), ("bf16", 8e-2)])
def test_f5_step_matches_oracle(vox, math, bar, pe_attn_head):
    B, N = 2, 40
    model = _model(1, **CFG)
    rng = np.random.default_rng(2)
    h = rng.standard_normal((B * N, CFG["D"])).astype(np.float32)
    ts = rng.standard_normal(CFG["D"]).astype(np.float32)
    plan = _plan(vox, _dev(*model), heads=CFG["H"], dim_head=CFG["HD"], batch=B, frames=N, pe_attn_head=pe_attn_head, math=math)
    out = plan.step(torch.from_numpy(h).cuda(), torch.from_numpy(ts).cuda()).cpu().numpy()
    h_after = plan.h.cpu().numpy()
    want, want_h = _oracle(model, h, ts, heads=CFG["H"], dim_head=CFG["HD"], batch=B, frames=N, pe_attn_head=pe_attn_head)
    plan.close()
    assert _rel(out, want) <= bar, _rel(out, want)
    assert _rel(h_after, want_h) <= bar, _rel(h_after, want_h)


@pytest.mark.parametrize("frames,pe_attn_head", [(70, 1), (128, 0), (300, 1), (520, 1)])
def test_f5_bf16_pipeline_matches_oracle(vox, frames, pe_attn_head):
    """dim_head 64 in bf16 mode: bf16 weight copies, fused q|k|v projection, the fused attention kernel (128-row query
    tiles, 64-key tiles; 70, 300 and 520 frames leave a ragged last tile of keys and of queries, 300 runs three query tiles
    and five key tiles, 520 nine key tiles: the key/value buffers rotate several times), residual and modulation fused."""
    cfg = dict(D=128, H=2, HD=64, FF=256, depth=2, out_dim=24)
    B = 2
    model = _model(6, **cfg)
    rng = np.random.default_rng(7)
    h = rng.standard_normal((B * frames, cfg["D"])).astype(np.float32)
    ts = rng.standard_normal(cfg["D"]).astype(np.float32)
    plan = _plan(vox, _dev(*model), heads=cfg["H"], dim_head=cfg["HD"], batch=B, frames=frames, pe_attn_head=pe_attn_head,
                 math="bf16")
    out = plan.step(torch.from_numpy(h).cuda(), torch.from_numpy(ts).cuda()).cpu().numpy()
    h_after = plan.h.cpu().numpy()
    want, want_h = _oracle(model, h, ts, heads=cfg["H"], dim_head=cfg["HD"], batch=B, frames=frames, pe_attn_head=pe_attn_head)
    plan.close()
    assert _rel(out, want) <= 8e-2, _rel(out, want)
    assert _rel(h_after, want_h) <= 8e-2, _rel(h_after, want_h)


@pytest.mark.parametrize("math,bar", [("f32", 2e-5), ("tf32", 2e-2), ("bf16", 8e-2)])
def test_f5_full_step_matches_reference_dit_forward(vox, golden, math, bar):
    """The whole dit_forward of the golden F5 model on the device: the input embedding (in_proj over [x, cond, temb],
    the two grouped position convolutions with Mish) in the same graph as the blocks and the output head."""
    from test_f5_oracle import f5_golden_model

    g = golden["f5"]
    dims, B, N, _, blocks = f5_golden_model(g)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()  # noqa: E731
    embed = {k: t(g[k]) for k in ("in_proj", "in_proj_b", "pos1_w", "pos1_b", "pos2_w", "pos2_b")}
    plan = vox.F5Dit([{k: t(v) for k, v in b.items()} for b in blocks], t(g["norm_out"]), t(g["proj_out"]), heads=dims["heads"],
                     dim_head=dims["dim_head"], batch=B, frames=N, pe_attn_head=dims["pe_attn_head"], math=math,
                     norm_out_b=t(g["norm_out_b"]), proj_out_b=t(g["proj_out_b"]), embed=embed)
    cond = np.concatenate([g["cond"], g["temb"]], axis=2)
    out = plan.step(None, t(g["ts"]), x=t(g["x"]), cond=t(cond)).cpu().numpy()
    plan.close()
    want = g["out"].reshape(B * N, -1).astype(np.float64)
    assert _rel(out, want) <= bar, _rel(out, want)


def test_f5_bf16_pipeline_with_embedding_matches_oracle(vox):
    cfg = dict(D=128, H=2, HD=64, FF=256, depth=2, out_dim=24)
    B, N, TD = 2, 70, 32
    model = _model(8, **cfg)
    rng = np.random.default_rng(9)
    D = cfg["D"]
    emb = {"in_proj": (rng.standard_normal((D, 2 * cfg["out_dim"] + TD)) * 0.1).astype(np.float32),
           "in_proj_b": (rng.standard_normal(D) * 0.1).astype(np.float32),
           "pos1_w": (rng.standard_normal((D, D // 16, 31)) / np.sqrt(31 * D // 16)).astype(np.float32),
           "pos1_b": (rng.standard_normal(D) * 0.1).astype(np.float32),
           "pos2_w": (rng.standard_normal((D, D // 16, 31)) / np.sqrt(31 * D // 16)).astype(np.float32),
           "pos2_b": (rng.standard_normal(D) * 0.1).astype(np.float32)}
    x = rng.standard_normal((B, N, cfg["out_dim"])).astype(np.float32)
    cond = rng.standard_normal((B, N, cfg["out_dim"])).astype(np.float32)
    temb = rng.standard_normal((B, N, TD)).astype(np.float32)
    ts = rng.standard_normal(D).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    plan = _plan(vox, _dev(*model), heads=cfg["H"], dim_head=cfg["HD"], batch=B, frames=N, math="bf16",
                 embed={k: t(v) for k, v in emb.items()})
    out = plan.step(None, t(ts), x=t(x), cond=t(np.concatenate([cond, temb], axis=2))).cpu().numpy()
    plan.close()
    h = F5.embed(x, cond, temb, emb["in_proj"], emb["in_proj_b"], emb["pos1_w"], emb["pos1_b"], emb["pos2_w"], emb["pos2_b"])
    want, _ = _oracle(model, h, ts, heads=cfg["H"], dim_head=cfg["HD"], batch=B, frames=N)
    assert _rel(out, want) <= 8e-2, _rel(out, want)


def test_f5_replay_is_deterministic_and_reads_fresh_inputs(vox):
    B, N = 2, 33
    model = _model(3, **CFG)
    plan = _plan(vox, _dev(*model), heads=CFG["H"], dim_head=CFG["HD"], batch=B, frames=N, math="f32")
    outs = []
    for seed in (0, 1, 0):
        r = np.random.default_rng(seed)
        h = r.standard_normal((B * N, CFG["D"])).astype(np.float32)
        ts = r.standard_normal(CFG["D"]).astype(np.float32)
        outs.append(plan.step(torch.from_numpy(h).cuda(), torch.from_numpy(ts).cuda()).cpu().numpy())
        if seed == 1:
            want, _ = _oracle(model, h, ts, heads=CFG["H"], dim_head=CFG["HD"], batch=B, frames=N)
            assert _rel(outs[-1], want) <= 2e-5
    np.testing.assert_array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))
    assert not np.array_equal(outs[0], outs[1])
    plan.close()


def test_f5_rejects_mismatched_weights(vox):
    blocks, norm_out, proj_out, _, _ = _dev(*_model(5, **CFG))
    blocks[0]["o"] = blocks[0]["o"][:, :-1].contiguous()
    with pytest.raises(vox.VoxCudaError) as e:
        vox.F5Dit(blocks, norm_out, proj_out, heads=CFG["H"], dim_head=CFG["HD"], batch=1, frames=8)
    assert e.value.status == -6
    blocks, norm_out, proj_out, _, _ = _dev(*_model(5, **CFG))
    blocks[1]["ff1_b"] = blocks[1]["ff1_b"][:-1].contiguous()
    with pytest.raises(vox.VoxCudaError) as e:
        vox.F5Dit(blocks, norm_out, proj_out, heads=CFG["H"], dim_head=CFG["HD"], batch=1, frames=8)
    assert e.value.status == -6
