"""TEST INFRASTRUCTURE — numpy restatement of the F5-TTS DiT transformer step. Not product code.

Follows Vox's CPU F5Model::dit_forward (src/f5.cpp:563-724): the input embedding (embed: in_proj and the convolutional
position embedding with Mish) and the blocks and output head (dit), in float64 except for the quantities the CPU builds in
float32 (the RoPE table, f5.cpp:529-541). Only tests/ and the CPU-baseline leg of bench.py use it.

Parity of the pieces is pinned elsewhere: the modulated LayerNorm (the adaLN modulate lambda, f5.cpp:617-632), GELU-tanh
(f5.cpp:93-96) and the row softmax against the reference compiled from its sources (tests/golden); the RoPE here is
the interleaved-pair rotation of f5.cpp:689-704. The composition itself is restated from f5.cpp and not pinned against
a run of the reference (that needs an F5 checkpoint).
"""

from __future__ import annotations

import numpy as np


def rope_table(frames: int, dim_head: int) -> tuple[np.ndarray, np.ndarray]:
    """(cos, sin) [frames][dim_head/2] as f5.cpp:529-541 builds them: inv in double then float, angle in float."""
    half = dim_head // 2
    inv = np.array([np.float32(1.0 / 10000.0 ** (2 * j / dim_head)) for j in range(half)], np.float32)
    ang = np.arange(frames, dtype=np.float32)[:, None] * inv[None, :]
    return np.cos(ang.astype(np.float64)).astype(np.float32), np.sin(ang.astype(np.float64)).astype(np.float32)


def modulate(x: np.ndarray, scale: np.ndarray, shift: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """LayerNorm without affine (mean and variance in double), then * (1 + scale) + shift (f5.cpp:617-632)."""
    mean = x.mean(axis=1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=1, keepdims=True)
    return (x - mean) / np.sqrt(var + eps) * (1.0 + scale[None, :]) + shift[None, :]


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """f5.cpp:93-96."""
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def rope(t: np.ndarray, frames: int, heads: int, dim_head: int, rope_heads: int) -> np.ndarray:
    """Rotates pairs (2j, 2j+1) of the first rope_heads heads at position r % frames (f5.cpp:689-704)."""
    R = t.shape[0]
    c, s = rope_table(frames, dim_head)
    pos = np.arange(R) % frames
    out = t.reshape(R, heads, dim_head // 2, 2).copy()
    x0, x1 = out[:, :rope_heads, :, 0].copy(), out[:, :rope_heads, :, 1].copy()
    cc, ss = c[pos][:, None, :].astype(np.float64), s[pos][:, None, :].astype(np.float64)
    out[:, :rope_heads, :, 0] = x0 * cc - x1 * ss
    out[:, :rope_heads, :, 1] = x1 * cc + x0 * ss
    return out.reshape(R, heads * dim_head)


def softmax(s: np.ndarray, scale: float) -> np.ndarray:
    """Row softmax of s * scale: max subtracted, exp, normalised (f5.cpp:651-661)."""
    s = np.asarray(s, np.float64) * scale
    e = np.exp(s - s.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, batch: int, frames: int, heads: int, dim_head: int) -> np.ndarray:
    """Per sequence and head: softmax(q k^T / sqrt(dim_head)) v, no mask (f5.cpp:635-668)."""
    shp = (batch, frames, heads, dim_head)
    qh, kh, vh = (a.reshape(shp).transpose(0, 2, 1, 3) for a in (q, k, v))
    p = softmax(qh @ kh.transpose(0, 1, 3, 2), float(np.float32(1.0) / np.sqrt(np.float32(dim_head))))
    return (p @ vh).transpose(0, 2, 1, 3).reshape(batch * frames, heads * dim_head)


def mish(x: np.ndarray) -> np.ndarray:
    """x tanh(softplus(x)), softplus = x past 20 (f5.cpp:97-100)."""
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    return x * np.tanh(sp)


def conv1d(x: np.ndarray, w: np.ndarray, b, groups: int) -> np.ndarray:
    """Grouped 1-D convolution over time of x [T][cin], weights [cout][cin/groups][K] (PyTorch layout), zero padding
    K/2 on both sides, + bias (Conv1d::forward, f5_ops.cpp:106-145)."""
    T, cin = x.shape
    cout, cig, K = w.shape
    cog, pad = cout // groups, K // 2
    xp = np.zeros((T + 2 * pad, cin))
    xp[pad:pad + T] = x
    y = np.zeros((T, cout))
    for g in range(groups):
        # windows [T][K][cig] of this group's channels
        win = np.stack([xp[k:k + T, g * cig:(g + 1) * cig] for k in range(K)], axis=1)
        wg = np.asarray(w[g * cog:(g + 1) * cog], np.float64)  # [cog][cig][K]
        y[:, g * cog:(g + 1) * cog] = np.einsum("tki,oik->to", win, wg)
    return y if b is None else y + np.asarray(b, np.float64)


def embed(x, cond, temb, in_proj, in_proj_b, pos1_w, pos1_b, pos2_w, pos2_b, groups: int = 16) -> np.ndarray:
    """The input embedding of dit_forward (f5.cpp:583-606): h = in_proj([x, cond, temb]) per row, then per sequence
    h += mish(conv2(mish(conv1(h)))). x, cond [B][N][mel], temb [B][N][text]; returns h [B*N][dim]."""
    B, N, _ = np.shape(x)
    cat = np.concatenate([np.asarray(x, np.float64), np.asarray(cond, np.float64), np.asarray(temb, np.float64)], axis=2)
    h = linear(cat.reshape(B * N, -1), in_proj, in_proj_b)
    for s in range(B):
        hs = h[s * N:(s + 1) * N]
        a = mish(conv1d(hs, pos1_w, pos1_b, groups))
        hs += mish(conv1d(a, pos2_w, pos2_b, groups))
    return h


def linear(x, w, b=None):
    """y = x W^T (+ b): Vox's matmul with the bias its Mat carries (kernels.hpp:83, f5.cpp:59-84)."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    return y if b is None else y + np.asarray(b, np.float64)


def dit(h, ts, blocks, norm_out, proj_out, *, heads: int, dim_head: int, batch: int, frames: int, pe_attn_head: int = 0,
        norm_out_b=None, proj_out_b=None):
    """Returns (out [R][out_dim], h after the blocks [R][D]) in float64 for h [R][D], ts [D] and the weights (numpy
    arrays, [out][in] as Vox's Mat, each with an optional bias "<name>_b"): the loop of f5.cpp:678-717 and the output of
    f5.cpp:719-723."""
    h = np.asarray(h, np.float64).copy()
    ts = np.asarray(ts, np.float64)
    D = h.shape[1]
    rope_heads = pe_attn_head if pe_attn_head > 0 else heads
    for L in blocks:
        lin = lambda x, k: linear(x, L[k], L.get(k + "_b"))  # noqa: E731
        ada = lin(ts[None, :], "ada")[0]
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (ada[i * D:(i + 1) * D] for i in range(6))
        nrm = modulate(h, scale_msa, shift_msa)
        q, k, v = lin(nrm, "q"), lin(nrm, "k"), lin(nrm, "v")
        q, k = rope(q, frames, heads, dim_head, rope_heads), rope(k, frames, heads, dim_head, rope_heads)
        at = attention(q, k, v, batch, frames, heads, dim_head)
        h += gate_msa[None, :] * lin(at, "o")
        nrm = modulate(h, scale_mlp, shift_mlp)
        ff = gelu_tanh(lin(nrm, "ff1"))
        h += gate_mlp[None, :] * lin(ff, "ff2")
    fin = linear(ts[None, :], norm_out, norm_out_b)[0]  # (scale, shift)
    out = linear(modulate(h, fin[:D], fin[D:]), proj_out, proj_out_b)
    return out, h
