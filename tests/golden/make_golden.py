"""Generate the golden fixtures of the Vox operator path from dariumi/Vox's own CPU code.

Inputs come from the seeded Philox generator of the C restatement (oracle/vox_oracle.c, itself checked against
the reference's DetRng and F5Model::noise in gen.npz); every output is computed by the reference library
oracle/_ref/libvox_ref.so, which is compiled from the reference sources (make -C oracle ref REF=...). The fixtures
let the tests pin the oracle and the CUDA kernels on machines where the reference sources are absent.

Run from the repository root: ``python tests/golden/make_golden.py``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.oracle import port, ref  # noqa: E402

OUT = Path(__file__).resolve().parent


def main() -> None:
    P, R = port(), ref()
    if R is None:
        raise SystemExit("oracle/_ref/libvox_ref.so is missing: build it with `make -C oracle ref REF=<reference root>`")

    # -- generator: DetRng::uniform and F5Model::noise of the reference
    frames = np.arange(256, dtype=np.uint64)
    uni = np.array([[[R.uniform(s, int(f), 7, d) for f in frames] for d in (0, 1)] for s in (0, 42)], np.float32)
    np.savez_compressed(OUT / "gen.npz", uniform_seeds=np.array([0, 42], np.uint64), uniform=uni,
                        noise_0_0=R.f5_noise(0, 0, 1001), noise_12345_3=R.f5_noise(12345, 3, 513))

    # -- normalisation
    x = P.normal((6, 1024))
    w = P.normal((1024,), 1.0, 0.02, sid=1)
    b = P.normal((1024,), 0.0, 0.1, sid=2)
    x33 = P.normal((3, 33), sid=7)
    X = P.normal((2, 8, 1024), sid=8)
    sh = P.normal((2, 1024), 0.0, 0.1, sid=3)
    sc = P.normal((2, 1024), 0.0, 0.1, sid=4)
    g = P.normal((2, 1024), 0.0, 0.1, sid=5)
    res = P.normal((2, 8, 1024), sid=6)
    np.savez_compressed(
        OUT / "norm.npz", x=x, w=w, b=b, x33=x33, X=X, shift=sh, scale=sc, gate=g, res=res,
        rmsnorm=R.rmsnorm(x, w, 1e-6), rmsnorm33=R.rmsnorm(x33, w[:33], 1e-6),
        layernorm=R.layernorm(x, w, b, 1e-5), layernorm_nob=R.layernorm(x, w, None, 1e-5),
        ln_modulate=R.nn_layer_norm(x, w, b, 1e-6, True), ln_plain=R.nn_layer_norm(x, None, None, 1e-6),
        adaln_gated=R.adaln(X, sh, sc, g, res), adaln_modulate=R.adaln(X, sh, sc))

    # -- softmax (Vox's causal composition of kernels.cpp:812-819)
    s = P.normal((2, 64, 64), 0.0, 3.0, sid=10)
    s2 = P.normal((2, 16, 40), 0.0, 3.0, sid=11)
    k = np.float32(1.0 / np.sqrt(128.0))
    np.savez_compressed(
        OUT / "softmax.npz", s=s, s2=s2, scale=k,
        causal=R.softmax_rows(s, k, 64, 0), full=R.softmax_rows(s, k, 0, 0),
        causal_pos24=R.softmax_rows(s2, k, 16, 24), causal_fast=R.softmax_rows(s, k, 64, 0, fast=True))

    # -- activations
    gg = P.normal((4, 3072), sid=20)
    uu = P.normal((4, 3072), sid=21)
    xg = P.normal((4099,), 0.0, 2.0, sid=22)
    al = P.uniform_arr((8,), 0.2, 2.0, sid=23)
    xs = P.normal((2, 8, 100), sid=24)
    ib = P.uniform_arr((8,), 0.5, 1.5, sid=25)
    np.savez_compressed(
        OUT / "act.npz", g=gg, u=uu, xg=xg, alpha=al, xs=xs, inv_b=ib,
        silu_mul=R.silu_mul(gg, uu), gelu_erf=R.gelu_erf(xg), gelu_inplace=R.gelu_inplace(xg), gelu_tanh=R.gelu_tanh(xg),
        snake_hift_cm=R.snake(xs, al, 0, inner=100), snake_hift_tm=R.snake(xs, al, 0, inner=1),
        snake_kokoro_cm=R.snake(xs, al, 2, inner=100), snake_kokoro_tm=R.snake(xs, al, 2, inner=1),
        snake_beta_tm=R.snake(xs, al, 1, ib, inner=1),
        fast_sin_x=np.linspace(-60, 60, 2001, dtype=np.float32),
        fast_sin=np.array([R.fast_sin(v) for v in np.linspace(-60, 60, 2001, dtype=np.float32)], np.float32))

    # -- block dequantisation (f16 scale bits converted by the reference's f16_to_f32)
    q8 = P.fill_i8((64, 256), -128, 127, sid=30)
    q4 = P.fill_u8((64, 128), sid=31)
    s16 = P.uniform_arr((64, 8), 0.001, 0.05, sid=32).astype(np.float16)
    s16_bits = s16.view(np.uint16)
    s32 = R.f16_to_f32(s16_bits)
    wq = P.normal((16, 256), 0.0, 0.05, sid=33)
    rq8, rs8 = R.quantize_q8(wq)
    rq4, rs4 = R.quantize_q4(wq)
    np.savez_compressed(
        OUT / "dequant.npz", q8=q8, q4=q4, scale_f16_bits=s16_bits, scale_f32=s32,
        q8_out=R.mat_rows(q8, s32), q4_out=R.mat_rows(q4, s32, q4=True),
        wq=wq, quant_q8=rq8, quant_q8_scale=rs8, quant_q8_out=R.mat_rows(rq8, rs8),
        quant_q4=rq4, quant_q4_scale=rs4, quant_q4_out=R.mat_rows(rq4, rs4, q4=True))

    # -- broadcast bias-add
    yb = P.normal((8, 100), sid=40)
    bb = P.normal((100,), sid=41)
    np.savez_compressed(OUT / "bias.npz", y=yb, b=bb, out=R.bias_add(yb, bb))
    # -- transformer elementwise chain: transformer_forward's per-token q/k step (vox::rmsnorm per head, then
    #    vox::rope_apply, kernels.cpp:797-803) and the residual update + RMSNorm (kernels.cpp:822-825, 833)
    heads, kv, hd, m, pos0 = 4, 2, 128, 5, 37
    qkv = P.normal((m, (heads + 2 * kv) * hd), sid=50)
    qn = P.normal((hd,), 1.0, 0.1, sid=51)
    kn = P.normal((hd,), 1.0, 0.1, sid=52)
    inv = R.rope_inv_freq(hd, 1e6)
    qs, ks = qkv[:, :heads * hd], qkv[:, heads * hd:(heads + kv) * hd]
    q_nrm, k_nrm = R.qk_norm_rope(qs, ks, qn, kn, inv, heads, kv, hd, pos0)
    q_raw, k_raw = R.qk_norm_rope(qs, ks, None, None, inv, heads, kv, hd, pos0)
    hh = P.normal((6, 1024), sid=53)
    dd = P.normal((6, 1024), sid=54)
    ls = P.normal((1024,), 0.0, 0.1, sid=55)
    wn = P.normal((1024,), 1.0, 0.02, sid=56)
    h_ls, xn_ls = R.add_rmsnorm(hh, dd, ls, wn)
    h_no, xn_no = R.add_rmsnorm(hh, dd, None, wn)
    np.savez_compressed(
        OUT / "xfmr.npz", qkv=qkv, qn=qn, kn=kn, inv_freq=inv, inv_freq_64=R.rope_inv_freq(64, 1e4),
        dims=np.array([heads, kv, hd, m, pos0], np.int64),
        q_norm_rope=q_nrm, k_norm_rope=k_nrm, q_rope=q_raw, k_rope=k_raw,
        h=hh, d=dd, ls=ls, w=wn, h_ls=h_ls, xn_ls=xn_ls, h_no=h_no, xn_no=xn_no)
    # -- quantized GEMV with float activations: the reference's own matmul, Q8 weights with m = 9 (its
    #    dequantise-then-f32 path, kernels.cpp:669-688) and the dequantised (mat_rows) weights as F32 for m <= 8 and Q4
    gr, gc = 48, 256
    gq8 = P.fill_i8((gr, gc), -127, 127, sid=100)
    gq4 = P.fill_u8((gr, gc // 2), sid=101)
    gs = P.uniform_arr((gr, gc // 32), 0.001, 0.05, sid=102)
    gb = P.normal((gr,), sid=103)
    gx = P.normal((9, gc), sid=104)
    np.savez_compressed(
        OUT / "gemv.npz", q8=gq8, q4=gq4, scale=gs, bias=gb, x=gx,
        q8_m9=R.matmul(3, gq8, gs, gx, gr, gc, gb),
        q8_m3=R.matmul(0, R.mat_rows(gq8, gs), None, gx[:3], gr, gc, gb),
        q4_m3=R.matmul(0, R.mat_rows(gq4, gs, q4=True), None, gx[:3], gr, gc, gb),
        q4_m1_nobias=R.matmul(0, R.mat_rows(gq4, gs, q4=True), None, gx[:1], gr, gc))
    # -- .tmod container written by the reference's own tmod_write (formats.cpp:215-249): Q8 and Q4 matrices with
    #    their f32 scales (nn::mat_named, nn.cpp:132-145), an f32 vector, a bf16 table; a manifest with nested values
    tq8 = P.fill_i8((48, 64), -127, 127, sid=130)
    tq4 = P.fill_u8((16, 32), sid=131)
    ts8 = P.uniform_arr((48, 2), 0.001, 0.05, sid=132)
    ts4 = P.uniform_arr((16, 2), 0.001, 0.05, sid=133)
    tnorm = P.normal((64,), 1.0, 0.02, sid=134)
    temb = P.bf16_round(P.normal((3, 8), sid=135))
    manifest = ('{"family": "test", "config": {"hidden": 64, "eps": 1e-06, "name": "\u00fcn\u00efcode \\"q\\" \\\\", '
                '"list": [1, 2.5, true, false, null, [], {}], "\u20ac": -3e2}}')
    R.tmod_write(OUT / "tiny.tmod", manifest, {
        "layer.w": (5, (48, 64), tq8.tobytes()), "layer.w.scale": (0, (48, 2), ts8.tobytes()),
        "layer.u": (6, (16, 32), tq4.tobytes()), "layer.u.scale": (0, (16, 2), ts4.tobytes()),
        "norm": (0, (64,), tnorm.tobytes()), "emb": (2, (3, 8), np.asarray(temb, np.uint16).tobytes())})
    np.savez_compressed(OUT / "tmod.npz", q8=tq8, q4=tq4, s8=ts8, s4=ts4, norm=tnorm, emb=np.asarray(temb, np.uint16),
                        q8_deq=R.mat_rows(tq8, ts8), q4_deq=R.mat_rows(tq4, ts4, q4=True))
    f5_golden(P, R)
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


# -- F5 DiT forward (F5Model::dit_forward, f5.cpp:563-724) of a tiny random model written with the reference's own
#    tmod_write: every linear with a bias, RoPE on the first head only (pe_attn_head 1), no text-encoder or Vocos
#    layers. Saved: the inputs, the weights of the input embedding (in_proj, the two grouped position convolutions),
#    of the blocks and of the output head, the reference's time embedding ts and its output.
F5_DIMS = dict(dim=32, depth=2, heads=2, dim_head=16, ff_mult=2, text_dim=16, text_rows=4, mel_dim=20, pe_attn_head=1)


def f5_golden(P, R) -> None:
    import json
    import tempfile

    c = F5_DIMS
    D, M, TD, L = c["dim"], c["mel_dim"], c["text_dim"], c["depth"]
    IN, FF = c["heads"] * c["dim_head"], c["ff_mult"] * c["dim"]
    sid = [300]

    def nrm(shape, std):
        sid[0] += 1
        return P.normal(shape, 0.0, std, sid=sid[0]).astype(np.float32)

    lin = lambda o, i: (nrm((o, i), 1.0 / np.sqrt(i)), nrm((o,), 0.1))  # noqa: E731
    blobs, arrays = {}, {}

    def put(name, arr):
        blobs[name] = (0, arr.shape, np.ascontiguousarray(arr, np.float32).tobytes())

    def put_lin(name, key, o, i):
        w, b = lin(o, i)
        put(name + ".weight", w)
        put(name + ".bias", b)
        if key:
            arrays[key], arrays[key + "_b"] = w, b

    put("mel.fb", np.abs(nrm((M, 9), 0.1)))  # n_fft 16
    d = "dit."
    put_lin(d + "time_embed.time_mlp.0", None, D, 256)
    put_lin(d + "time_embed.time_mlp.2", None, D, D)
    put(d + "text_embed.text_embed.weight", nrm((c["text_rows"], TD), 1.0))
    put_lin(d + "input_embed.proj", "in_proj", D, 2 * M + TD)
    for j in (0, 2):  # grouped (16) position convolutions, kernel 31
        w, b = nrm((D, D // 16, 31), 1.0 / np.sqrt(31 * D // 16)), nrm((D,), 0.1)
        put(d + f"input_embed.conv_pos_embed.conv1d.{j}.weight", w)
        put(d + f"input_embed.conv_pos_embed.conv1d.{j}.bias", b)
        arrays[f"pos{j // 2 + 1}_w"], arrays[f"pos{j // 2 + 1}_b"] = w, b
    names = {"ada": "attn_norm.linear", "q": "attn.to_q", "k": "attn.to_k", "v": "attn.to_v", "o": "attn.to_out.0",
             "ff1": "ff.ff.0.0", "ff2": "ff.ff.2"}
    shapes = {"ada": (6 * D, D), "q": (IN, D), "k": (IN, D), "v": (IN, D), "o": (D, IN), "ff1": (FF, D), "ff2": (D, FF)}
    for l in range(L):
        for k, nm in names.items():
            put_lin(f"{d}transformer_blocks.{l}.{nm}", f"b{l}_{k}", *shapes[k])
    put_lin(d + "norm_out.linear", "norm_out", 2 * D, D)
    put_lin(d + "proj_out", "proj_out", M, D)
    V = 16
    put("vocos.backbone.embed.weight", nrm((V, M, 7), 0.1))
    for nm in ("norm", "final_layer_norm"):
        put(f"vocos.backbone.{nm}.weight", np.ones(V, np.float32))
        put(f"vocos.backbone.{nm}.bias", np.zeros(V, np.float32))
    put("vocos.head.out.weight", nrm((18, V), 0.1))
    manifest = {"family": "f5", "f5": {
        "dim": D, "depth": L, "heads": c["heads"], "dim_head": c["dim_head"], "ff_mult": c["ff_mult"], "text_dim": TD,
        "text_rows": c["text_rows"], "mel_dim": M, "conv_layers": 0, "pe_attn_head": c["pe_attn_head"],
        "mel": {"sample_rate": 24000, "n_fft": 16, "hop": 4, "win": 16, "n_mels": M},
        "vocos": {"dim": V, "intermediate": 32, "layers": 0, "n_fft": 16, "hop": 4, "padding": "same"},
        "tokenizer": {"type": "char", "vocab": ["a"]}}}
    B, N, t = 2, 24, 0.37
    x, cond, temb = nrm((B, N, M), 1.0), nrm((B, N, M), 1.0), nrm((B, N, TD), 1.0)
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "f5.tmod"
        R.tmod_write(path, json.dumps(manifest), blobs)
        ts, out = R.f5_dit(path, x, cond, temb, t, D)
    np.savez_compressed(OUT / "f5.npz", dims=np.array([c[k] for k in F5_DIMS], np.int64), x=x, cond=cond, temb=temb,
                        t=np.float32(t), ts=ts, out=out, **arrays)


if __name__ == "__main__":
    main()
