#!/usr/bin/env python3
"""Benchmark of the Vox memory-bound operator path on B200 (one JSON line on rank 0).

A step is one pass of the whole hot path over one batch of synthetic input at BASELINE's shapes ("vox-hotpath-suite"):
  cfg1  RMSNorm x[512,1024] f32 (eps 1e-6, w ~N(1,0.02)) and SwiGLU silu(g)*u, g,u [512,3072] f32
  cfg2  causal scaled softmax, scores [16,1024,1024] f32 ~N(0,3) x 1/sqrt(128)
  cfg3  fused adaLN block, x/residual [8,2048,1024] bf16, shift/scale/gate [8,1024] bf16, eps 1e-6
  cfg4  q8 and q4 dequant [4096,4096] (f16 scales, block 32) -> bf16; HiFT Snake x [16,512,24000] f32
  cfg5  sweep per GPU: add / mul / GELU / row sum / row max / row L2 (rows of 4096) in f32 and bf16 over
        --sweep-elems elements each, plus the deterministic global sum of the f32 tensor across all ranks
        (slot partials -> one NCCL all-reduce of 840 f64 -> fixed-order fold).
value = algorithmic bytes of all ranks (each input read once, each output written once) / step time (max over
ranks, CUDA events). Scaling is weak: every rank runs the full per-GPU suite on its own shard of a global batch
(inputs drawn from Philox counters offset by the rank), and only the global sum exchanges data.

--impl reference times dariumi/Vox's own CPU operators (oracle/_ref/libvox_ref.so, compiled from the reference
sources; the C restatement if that library is absent) on the host cores over a bounded sample of the same suite.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "HBM GB/s & % of B200 peak per op; elements/s at 1/2/4/8 GPUs vs host CPU"
FALLBACK_HBM_GBS = 6650.0  # used only if MEASURED_PEAKS.json is absent
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0  # ditto


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops_sustained"]), "measured"
        except Exception:
            pass
    return FALLBACK_BF16_TFLOPS_SUSTAINED, "fallback"


# ---------------------------------------------------------------------------------------------------- workload

class Suite:
    """Device buffers and the per-op launch list of one step. `ops` entries: (name, bytes, elements, fn).

    `only` (a regex) keeps the matching ops and allocates only their buffers (profiling of one kernel)."""

    def __init__(self, vox, torch, rank: int, world: int, sweep_elems: int, dist=None, only: str | None = None, scale: int = 1):
        import re

        self.vox, self.t, self.rank, self.world, self.dist = vox, torch, rank, world, dist
        dev = torch.device("cuda", torch.cuda.current_device())
        f32, bf16 = torch.float32, torch.bfloat16
        E = lambda *s, dt=f32: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        seed, c0 = 0, rank << 36  # shard k draws counters offset by k * 2^36: independent shards of one global batch
        fill = lambda t, d, a, b, sid: vox.fill_philox(t, d, a, b, seed=seed, stream_id=sid, counter0=c0)  # noqa: E731
        want = (lambda nm: re.search(only, nm) is not None) if only else (lambda nm: True)
        ops, self.io, self.flops, self.f5_plans = [], [], {}, []

        def add(name, nbytes, elems, fn, reads, writes, flops=None):
            ops.append((name, nbytes, elems, fn))
            self.io.append((reads, writes))
            if flops:
                self.flops[name] = flops

        # `scale` multiplies the rows / heads / batches of cfg1-cfg4 (1 = BASELINE's shapes; larger values measure the
        # kernels where their size does not limit them)
        K = scale
        # cfg1
        if want("cfg1_rmsnorm_f32"):
            m1 = 512 * K
            x1, w1, y1 = fill(E(m1, 1024), 1, 0, 1, 1), fill(E(1024), 1, 1, 0.02, 2), E(m1, 1024)
            add("cfg1_rmsnorm_f32", 2 * m1 * 1024 * 4 + 1024 * 4, m1 * 1024, lambda: vox.rmsnorm(x1, w1, 1e-6, out=y1), [x1, w1], [y1])
        if want("cfg1_swiglu_f32"):
            m1 = 512 * K
            g1, u1, h1 = fill(E(m1, 3072), 1, 0, 1, 3), fill(E(m1, 3072), 1, 0, 1, 4), E(m1, 3072)
            add("cfg1_swiglu_f32", 3 * m1 * 3072 * 4, m1 * 3072, lambda: vox.silu_mul(g1, u1, out=h1), [g1, u1], [h1])
        # cfg2
        if want("cfg2_softmax_causal_f32"):
            H2 = 16 * K
            s2, p2 = fill(E(H2, 1024, 1024), 1, 0, 3, 5), E(H2, 1024, 1024)
            sc2 = float(1.0 / np.sqrt(128.0))
            add("cfg2_softmax_causal_f32", H2 * 1024 * 1025 // 2 * 4 + H2 * 1024 * 1024 * 4, H2 * 1024 * 1024,
                lambda: vox.softmax_rows(s2, sc2, 1024, 0, out=p2), [s2], [p2])
        # cfg3
        if want("cfg3_adaln_bf16"):
            B, T, D = 8 * K, 2048, 1024
            x3, r3, y3 = fill(E(B, T, D, dt=bf16), 1, 0, 1, 6), fill(E(B, T, D, dt=bf16), 1, 0, 1, 7), E(B, T, D, dt=bf16)
            sh3, sc3, g3 = (fill(E(B, D, dt=bf16), 1, 0, 0.1, s) for s in (8, 9, 10))
            add("cfg3_adaln_bf16", 3 * B * T * D * 2 + 3 * B * D * 2, B * T * D, lambda: vox.adaln(x3, sh3, sc3, 1e-6, g3, r3, out=y3),
                [x3, r3, sh3, sc3, g3], [y3])
        # cfg4
        R4 = 4096 * K
        if want("cfg4_dequant_q8_bf16") or want("cfg4_dequant_q4_bf16"):
            s4 = fill(E(R4, 128), 0, 0.001, 0.05, 13).to(torch.float16)
        if want("cfg4_dequant_q8_bf16"):
            q8, o8 = fill(E(R4, 4096, dt=torch.int8), 2, -128, 127, 11), E(R4, 4096, dt=bf16)
            add("cfg4_dequant_q8_bf16", R4 * 4096 + R4 * 128 * 2 + R4 * 4096 * 2, R4 * 4096,
                lambda: vox.dequant_q8(q8, s4, out=o8), [q8, s4], [o8])
        if want("cfg4_dequant_q4_bf16"):
            q4, o4 = fill(E(R4, 2048, dt=torch.uint8), 3, 0, 0, 12), E(R4, 4096, dt=bf16)
            add("cfg4_dequant_q4_bf16", R4 * 2048 + R4 * 128 * 2 + R4 * 4096 * 2, R4 * 4096,
                lambda: vox.dequant_q4(q4, s4, out=o4), [q4] + ([] if want("cfg4_dequant_q8_bf16") else [s4]), [o4])
        if want("cfg4_snake_hift_f32"):
            B4 = 16 * K
            xs, al, ys = fill(E(B4, 512, 24000), 1, 0, 1, 14), fill(E(512), 0, 0.2, 2.0, 15), E(B4, 512, 24000)
            add("cfg4_snake_hift_f32", 2 * B4 * 512 * 24000 * 4 + 512 * 4, B4 * 512 * 24000,
                lambda: vox.snake(xs, al, vox.SNAKE_HIFT, out=ys), [xs, al], [ys])
        # next rows of the path (not in the default suite; selected by name with --only next_): the transformer
        # elementwise chain on a Qwen3-0.6B-shaped prefill chunk (16 q / 8 kv heads of 128, hidden 1024)
        want_next = (lambda nm: re.search(only, nm) is not None) if only else (lambda nm: False)
        if want_next("next_qkv_rope_f32"):
            mt, nh, nkv, hd = 8192 * K, 16, 8, 128
            qkv = fill(E(mt, (nh + 2 * nkv) * hd), 1, 0, 1, 20)
            qn, kn = fill(E(hd), 1, 1, 0.1, 21), fill(E(hd), 1, 1, 0.1, 22)
            cs = vox.rope_table(vox.rope_inv_freq(hd, 1e6, device=dev), 0, mt)
            qo, kc, vc = E(mt, nh * hd), E(mt, nkv * hd), E(mt, nkv * hd)
            nb = 2 * mt * (nh + 2 * nkv) * hd * 4 + mt * hd * 4 + 2 * hd * 4
            add("next_qkv_rope_f32", nb, mt * (nh + 2 * nkv) * hd,
                lambda: vox.qkv_rope(qkv, cs, nh, nkv, hd, kc, vc, 0, q_norm_w=qn, k_norm_w=kn, q=qo), [qkv, cs, qn, kn], [qo, kc, vc])
        if want_next("next_add_rmsnorm_f32"):
            mt, H = 8192 * K, 1024
            hh, dd, wn, xo = fill(E(mt, H), 1, 0, 1, 23), fill(E(mt, H), 1, 0, 1, 24), fill(E(H), 1, 1, 0.02, 25), E(mt, H)
            add("next_add_rmsnorm_f32", 4 * mt * H * 4 + H * 4, mt * H, lambda: vox.add_rmsnorm(hh, dd, wn, 1e-6, out=xo), [hh, dd, wn],
                [hh, xo])
        # quantized decode GEMV (y = W x, m activation rows): Qwen3-8B MLP-up-shaped weights [12288][4096] with f16
        # scales, rotated over enough matrices that the weights stream from HBM (> 126 MB L2) on every call
        for qt in ("q8", "q4"):
            names = [f"next_gemv_{qt}_m{mm}" for mm in (1, 4, 8)]
            if not any(want_next(nm) for nm in names):
                continue
            GR, GC = 12288 * K, 4096
            nmat = 4 if qt == "q8" else 8
            if qt == "q8":
                mats = [fill(E(GR, GC, dt=torch.int8), 2, -128, 127, 26 + i) for i in range(nmat)]
            else:
                mats = [fill(E(GR, GC // 2, dt=torch.uint8), 3, 0, 0, 26 + i) for i in range(nmat)]
            scs = [fill(E(GR, GC // 32), 0, 0.001, 0.05, 40 + i).to(torch.float16) for i in range(nmat)]
            gx = fill(E(8, GC), 1, 0, 1, 50)
            gy = E(8, GR)
            fn = vox.gemv_q8 if qt == "q8" else vox.gemv_q4
            wbytes = GR * GC if qt == "q8" else GR * GC // 2
            for mm in (1, 4, 8):
                nm = f"next_gemv_{qt}_m{mm}"
                if not want_next(nm):
                    continue
                ctr = [0]

                def call(fn=fn, mats=mats, scs=scs, mm=mm, ctr=ctr):
                    i = ctr[0] % len(mats)
                    ctr[0] += 1
                    fn(mats[i], scs[i], gx[:mm], out=gy[:mm])

                add(nm, wbytes + GR * (GC // 32) * 2 + mm * GC * 4 + mm * GR * 4, GR * GC * mm, call, [mats[0], scs[0], gx], [gy])
        # F5-TTS DiT step (gpu_f5_step as one CUDA graph: input embedding, 22 blocks, output head): F5 base (dim 1024, 16
        # heads x 64, ff 2048, mel 100, text 512) on 2 sequences (conditional and unconditional) of 1024 frames, seeded
        # random weights and biases; each step writes x, the condition and the time embedding into the plan, then replays
        if any(want_next(f"next_f5_dit_{m}") for m in ("tf32", "bf16")):
            D, H, HD, FFm, L, O, Bq, Nf = 1024, 16, 64, 2, 22, 100, 2, 1024
            IN, FF, Rr = H * HD, FFm * D, Bq * Nf
            gen = torch.Generator(device=dev).manual_seed(7)
            W = lambda o, i, s=1.0: torch.randn(o, i, device=dev, generator=gen) * (s * i ** -0.5)  # noqa: E731
            Bv = lambda o: torch.randn(o, device=dev, generator=gen) * 0.1  # noqa: E731
            fblocks = []
            for _ in range(L):  # every linear biased, as F5 checkpoints are
                fb = {"ada": W(6 * D, D, 0.3), "q": W(IN, D), "k": W(IN, D), "v": W(IN, D), "o": W(D, IN), "ff1": W(FF, D), "ff2": W(D, FF)}
                fb.update({k + "_b": Bv(fb[k].shape[0]) for k in list(fb)})
                fblocks.append(fb)
            norm_out, proj_out, norm_out_b, proj_out_b = W(2 * D, D, 0.3), W(O, D), Bv(2 * D), Bv(O)
            TDm, KP = 512, 31  # text_dim, position-convolution kernel
            IND = 2 * O + TDm
            Wc = lambda: torch.randn(D, D // 16, KP, device=dev, generator=gen) * ((KP * D // 16) ** -0.5)  # noqa: E731
            fembed = {"in_proj": W(D, IND), "in_proj_b": Bv(D), "pos1_w": Wc(), "pos1_b": Bv(D), "pos2_w": Wc(), "pos2_b": Bv(D)}
            x0, cond0, ts0 = fill(E(Rr, O), 1, 0, 1, 60), fill(E(Rr, IND - O), 1, 0, 1, 62), fill(E(D), 1, 0, 1, 61)
            fl = L * (2 * 6 * D * D + 3 * 2 * Rr * D * IN + 2 * 2 * Bq * H * Nf * Nf * HD + 2 * Rr * IN * D + 2 * 2 * Rr * D * FF) \
                + 2 * 2 * D * D + 2 * Rr * D * O + 2 * Rr * D * IND + 2 * 2 * Rr * D * (D // 16) * KP
            wbytes = 4 * (L * (6 * D * D + 4 * D * IN + 2 * D * FF) + 2 * D * D + O * D + D * IND + 2 * D * (D // 16) * KP)
            for m in ("tf32", "bf16"):
                nm = f"next_f5_dit_{m}"
                if not want_next(nm):
                    continue
                plan = vox.F5Dit(fblocks, norm_out, proj_out, heads=H, dim_head=HD, batch=Bq, frames=Nf, math=m, norm_out_b=norm_out_b,
                                 proj_out_b=proj_out_b, embed=fembed)
                self.f5_plans.append(plan)

                def f5_step(plan=plan):
                    plan.x.copy_(x0)
                    plan.cond.copy_(cond0)
                    plan.ts.copy_(ts0)
                    plan.run()

                add(nm, wbytes + (Rr * IND + D + Rr * O) * 4, Rr, f5_step, [x0, cond0, ts0], [plan.out], flops=fl)
        # .tmod -> device: a file of Q8 matrices with f32 scales (Qwen3-8B MLP-shaped, [12288][4096] each, about 1.6 GB in
        # all), written once to a temporary directory; one step uploads every blob from the mapped file (page cache)
        if want_next("next_tmod_upload"):
            import tempfile

            from vox_b200.tmodfile import write_tmod

            tdir = Path(tempfile.mkdtemp(prefix="vox_tmod_"))
            TR, TC, TN = 12288, 4096, 4
            gen = np.random.default_rng(11)
            blobs = {}
            for i in range(TN):
                blobs[f"l{i}.w"] = ("I8", (TR, TC), gen.integers(-128, 128, (TR, TC), dtype=np.int8).tobytes())
                blobs[f"l{i}.w.scale"] = ("F32", (TR, TC // 32), gen.random((TR, TC // 32), dtype=np.float32).tobytes())
            write_tmod(tdir / "bench.tmod", {"family": "bench"}, blobs)
            nbytes = sum(len(b[2]) for b in blobs.values())
            del blobs
            self.tmod = vox.Tmod(tdir / "bench.tmod")
            tnames = self.tmod.names()
            touts = [E(*self.tmod.info(nm)[1], dt=torch.int8 if nm.endswith(".w") else torch.float32) for nm in tnames]
            add("next_tmod_upload", nbytes, nbytes, lambda: self.tmod.upload(tnames, touts), [], touts)
        # cfg5 sweep
        n = sweep_elems
        rows = n // 4096
        self.gsum_x = None
        for dt, tag, es in ((f32, "f32", 4), (bf16, "bf16", 2)):
            names = [f"cfg5_{k}_{tag}" for k in ("add", "mul", "gelu", "rowsum", "rowmax", "rowl2")]
            if es == 4:
                names.append("cfg5_global_sum_f32")
            if not any(want(nm) for nm in names):
                continue
            a = fill(E(rows, 4096, dt=dt), 1, 0, 1, 16 if es == 4 else 17)
            b = fill(E(rows, 4096, dt=dt), 1, 0, 1, 18 if es == 4 else 19)
            y, rr = E(rows, 4096, dt=dt), E(rows)
            if want(f"cfg5_add_{tag}"):
                add(f"cfg5_add_{tag}", 3 * n * es, n, lambda a=a, b=b, y=y: vox.add(a, b, out=y), [a, b], [y])
            if want(f"cfg5_mul_{tag}"):
                add(f"cfg5_mul_{tag}", 3 * n * es, n, lambda a=a, b=b, y=y: vox.mul(a, b, out=y), [a, b], [y])
            if want(f"cfg5_gelu_{tag}"):
                add(f"cfg5_gelu_{tag}", 2 * n * es, n, lambda a=a, y=y: vox.gelu(a, vox.GELU_ERF, out=y), [a], [y])
            for op, nm in ((vox.REDUCE_SUM, "rowsum"), (vox.REDUCE_MAX, "rowmax"), (vox.REDUCE_L2, "rowl2")):
                if want(f"cfg5_{nm}_{tag}"):
                    add(f"cfg5_{nm}_{tag}", n * es + rows * 4, n, lambda a=a, op=op, rr=rr: vox.row_reduce(a, op, out=rr), [a], [rr])
            if es == 4 and want("cfg5_global_sum_f32"):
                from vox_b200.shard import shard_rows

                self.gsum_x = a
                self.g_rows_total = rows * world
                self.g_row0, _ = shard_rows(self.g_rows_total, world, rank)
                self.slots, self.gscratch, self.gout = E(840, dt=torch.float64), E(rows), E(1, dt=torch.float64)
                add("cfg5_global_sum_f32", n * 4 + rows * 4, n, self.global_sum, [a], [self.gout])
        self.ops = ops
        self.kernels = {nm: (3 if nm == "cfg5_global_sum_f32" else 1) for nm, *_ in ops}
        self.bytes_per_step = sum(o[1] for o in ops)
        self.elems_per_step = sum(o[2] for o in ops)
        self.launches_per_step = sum(self.kernels.values())
        self.copy_in, self.copy_out = self.copy_plan(range(len(ops)))
        self.inputs = [t for c in self.copy_in for t in c]
        self.outputs = [t for c in self.copy_out for t in c]

    def copy_plan(self, order):
        """For ops run in `order`: the tensors to copy in before each op (first reader) and out after it (last writer)."""
        seen, last_w = set(), {}
        cin, cout = [], []
        for pos, i in enumerate(order):
            reads, writes = self.io[i]
            cin.append([t for t in reads if id(t) not in seen and not seen.add(id(t))])
            cout.append([])
            for t in writes:
                last_w[id(t)] = (pos, t)
        for pos, t in last_w.values():
            cout[pos].append(t)
        return cin, cout

    def e2e_order(self):
        """Op order for the host-buffer run: groups of ops that share tensors (cfg1 .. cfg5 f32 / bf16) ordered by
        Johnson's rule for a two-stage flow shop (copy-in, then copy-out): groups that copy in less than they copy out
        first, by increasing copy-in bytes; then the others by decreasing copy-out bytes. This shortens the copy-out
        tail after the last copy-in."""
        def group(name):
            if name.startswith("cfg5"):
                return "cfg5_" + name.rsplit("_", 1)[1]
            if name.startswith("cfg4_dequant"):
                return "cfg4_dequant"
            return name.split("_")[0] + ("_snake" if "snake" in name else "")
        groups = {}
        for i, (name, *_) in enumerate(self.ops):
            groups.setdefault(group(name), []).append(i)
        sized = []
        for g, idx in groups.items():
            cin, cout = self.copy_plan(idx)
            nbytes = lambda ts: sum(t.numel() * t.element_size() for c in ts for t in c)  # noqa: E731
            sized.append((g, idx, nbytes(cin), nbytes(cout)))
        first = sorted([x for x in sized if x[2] <= x[3]], key=lambda x: x[2])
        last = sorted([x for x in sized if x[2] > x[3]], key=lambda x: -x[3])
        return [i for _, idx, _, _ in first + last for i in idx]

    def global_sum(self):
        v = self.vox
        v.global_sum_partials(self.gsum_x, self.g_row0, self.g_rows_total, slots=self.slots, scratch=self.gscratch)
        if self.world > 1:
            self.dist.all_reduce(self.slots)
        v.global_sum_finish(self.slots, out=self.gout)

    def step(self, events=None):
        for i, (_, _, _, fn) in enumerate(self.ops):
            if events is not None:
                events[i][0].record()
            fn()
            if events is not None:
                events[i][1].record()


# ---------------------------------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples (200 ms) during the timed region: median SM MHz under load and throttle reasons."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx, self.proc, self.lines = gpu_index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------- CPU reference

def cpu_suite_sample(scale: float = 1.0):
    """Bounded sample of the suite on the host, through the reference's own CPU operators. Returns (lib, kind, cores, ops)
    with ops = [(name, bytes, elements, fn)]; byte model identical to the GPU arm's."""
    from oracle.oracle import port, ref

    R = ref()
    P = port()
    kind = "reference" if R is not None else "port"
    if R is not None:
        cores = R.set_threads(0)
    else:
        cores = 1
    L = R if R is not None else P
    f32 = np.float32
    ops = []
    x1, w1 = P.normal((512, 1024), sid=1), P.normal((1024,), 1, 0.02, sid=2)
    g1, u1 = P.normal((512, 3072), sid=3), P.normal((512, 3072), sid=4)
    ops.append(("cfg1_rmsnorm_f32", 2 * 512 * 1024 * 4 + 1024 * 4, 512 * 1024, lambda: L.rmsnorm(x1, w1, 1e-6)))
    ops.append(("cfg1_swiglu_f32", 3 * 512 * 3072 * 4, 512 * 3072, lambda: L.silu_mul(g1, u1)))
    hs = max(1, int(16 * scale))
    s2 = P.normal((hs, 1024, 1024), 0, 3, sid=5)
    ops.append(("cfg2_softmax_causal_f32", hs * (1024 * 1025 // 2 * 4 + 1024 * 1024 * 4), hs * 1024 * 1024,
                lambda: L.softmax_rows(s2, float(1 / np.sqrt(128.0)), 1024, 0)))
    Bs = max(1, int(8 * scale))
    x3 = P.normal((Bs, 2048, 1024), sid=6)
    r3 = P.normal((Bs, 2048, 1024), sid=7)
    sh3, sc3, g3 = (P.normal((Bs, 1024), 0, 0.1, sid=s) for s in (8, 9, 10))
    ops.append(("cfg3_adaln_bf16", Bs * (3 * 2048 * 1024 * 2 + 3 * 1024 * 2), Bs * 2048 * 1024,
                lambda: L.adaln(x3, sh3, sc3, g3, r3)))
    q8 = P.fill_i8((4096, 4096), -128, 127, sid=11)
    q4 = P.fill_u8((4096, 2048), sid=12)
    s4 = P.f16_to_f32(P.uniform_arr((4096, 128), 0.001, 0.05, sid=13).astype(np.float16).view(np.uint16))
    if R is not None:
        ops.append(("cfg4_dequant_q8_bf16", 4096 * 4096 * 3 + 4096 * 128 * 2, 4096 * 4096, lambda: P.bf16_round(R.mat_rows(q8, s4))))
        ops.append(("cfg4_dequant_q4_bf16", 4096 * 2048 + 4096 * 4096 * 2 + 4096 * 128 * 2, 4096 * 4096,
                    lambda: P.bf16_round(R.mat_rows(q4, s4, q4=True))))
    else:
        ops.append(("cfg4_dequant_q8_bf16", 4096 * 4096 * 3 + 4096 * 128 * 2, 4096 * 4096, lambda: P.bf16_round(P.dequant_q8(q8, s4))))
        ops.append(("cfg4_dequant_q4_bf16", 4096 * 2048 + 4096 * 4096 * 2 + 4096 * 128 * 2, 4096 * 4096,
                    lambda: P.bf16_round(P.dequant_q4(q4, s4))))
    Cs = max(4, int(512 * scale / 8))  # snake rows sampled: one batch, Cs channels
    xs, al = P.normal((1, Cs, 24000), sid=14), P.uniform_arr((Cs,), 0.2, 2.0, sid=15)
    ops.append(("cfg4_snake_hift_f32", 2 * Cs * 24000 * 4 + Cs * 4, Cs * 24000, lambda: L.snake(xs, al, 0, inner=24000)))
    n = int(2 ** 24 * scale)
    a, b = P.normal((n // 4096, 4096), sid=16), P.normal((n // 4096, 4096), sid=18)
    ops.append(("cfg5_add_f32", 3 * n * 4, n, lambda: L.add(a, b)))
    ops.append(("cfg5_mul_f32", 3 * n * 4, n, lambda: L.mul(a, b)))
    ops.append(("cfg5_gelu_f32", 2 * n * 4, n, (lambda: R.gelu_inplace(a)) if R is not None else (lambda: P.gelu(a, 0))))
    if R is not None:
        for op, nm in ((0, "rowsum"), (1, "rowmax"), (2, "rowl2")):
            ops.append((f"cfg5_{nm}_f32", n * 4 + n // 1024, n, lambda op=op: R.row_reduce(a, op)))
    else:
        for op, nm in ((0, "rowsum"), (1, "rowmax"), (2, "rowl2")):
            ops.append((f"cfg5_{nm}_f32", n * 4 + n // 1024, n, lambda op=op: P.row_reduce(a, op)))
    return kind, cores, ops, f32


def time_cpu(ops, reps: int = 1) -> tuple[float, int, int, dict]:
    """Seconds, bytes and elements over `reps` passes of the sampled suite (after one untimed pass)."""
    for *_, fn in ops:
        fn()
    per = {}
    t0 = time.perf_counter()
    for _ in range(reps):
        for nm, by, el, fn in ops:
            s = time.perf_counter()
            fn()
            per[nm] = per.get(nm, 0.0) + time.perf_counter() - s
    dt = time.perf_counter() - t0
    return dt, reps * sum(o[1] for o in ops), reps * sum(o[2] for o in ops), per


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    kind, cores, ops, _ = cpu_suite_sample(1.0)
    for _ in range(args.warmup):
        for *_, fn in ops:
            fn()
    dt, by, el, per = time_cpu(ops, reps=args.steps)
    value = by / dt / 1e9
    sample = ("per step: cfg1-cfg4 at BASELINE shapes except Snake on 64 of 8192 rows; cfg5 f32 add/mul/GELU/row "
              "sum/max/L2 on 2^24 elements; bf16 ops computed in f32 and rounded")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (Philox4x32-10 seed 0, BASELINE shapes)",
        "config": {"workload": "vox-hotpath-suite", "sample": sample},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "elements_per_s": round(el / dt, 1),
        "ops": {nm: {"gb_s": round(b * args.steps / per[nm] / 1e9, 3)} for nm, b, _, _ in ops},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------- GPU arm

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    import vox_b200 as vox

    suite = Suite(vox, torch, rank, world, args.sweep_elems, dist if world > 1 else None, only=args.only, scale=args.scale)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        suite.step()
    barrier()

    # The host enqueues launches while a spin kernel holds the GPU (torch.cuda._sleep, outside the timed region), so
    # the timed kernels run back to back and no host launch latency is timed.
    def prime(ms_guess: float):
        torch.cuda._sleep(int(min(max(ms_guess, 5.0), 2000.0) * 2.0e6))

    enqueue_ms = 0.08 * len(suite.ops)  # generous host cost of one step's launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        prime(enqueue_ms * args.steps)
        t0.record()
        for k in range(args.steps):
            suite.step()
        t1.record()
        barrier()
    ms = t0.elapsed_time(t1)
    # per-op breakdown: a second pass with an event pair around every launch
    nsteps_op = max(1, min(args.steps, 50))
    nops = len(suite.ops)
    ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(nops)] for _ in range(nsteps_op)]
    barrier()
    prime(enqueue_ms * 2 * nsteps_op)
    for k in range(nsteps_op):
        suite.step(ev[k])
    barrier()
    per_op = np.array([[ev[k][i][0].elapsed_time(ev[k][i][1]) for i in range(nops)] for k in range(nsteps_op)])  # ms
    op_ms = per_op.mean(0)
    times = torch.tensor([ms] + list(op_ms), dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, op_ms = float(times[0]), times[1:].cpu().numpy()

    # end to end through the public API with host buffers: pinned H2D of every input, the suite, D2H of every output
    e2e = run_e2e(suite, torch, dist, world, max(1, min(args.steps, args.e2e_steps))) if args.e2e_steps > 0 else None

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = peaks()
    step_s = ms / 1e3 / args.steps
    value = suite.bytes_per_step * world / step_s / 1e9
    ops = {}
    for (nm, by, el, _), t in zip(suite.ops, op_ms):
        gbs = by / (t / 1e3) / 1e9
        ops[nm] = {"us": round(t * 1e3, 2), "gb_s": round(gbs, 1), "frac_of_peak": round(gbs / peak, 3),
                   "elements_per_s": round(el / (t / 1e3), 1), "bytes": by}
        if nm in suite.flops:  # tensor-core rows: against the measured bf16 GEMM peak (sustained: a long step)
            tf = suite.flops[nm] / (t / 1e3) / 1e12
            tpk, tkind = tensor_peak()
            ops[nm].update({"tflops": round(tf, 1), "flops": suite.flops[nm], "frac_of_tensor_peak": round(tf / tpk, 3),
                            "tensor_peak": f"{tpk} TFLOP/s bf16 sustained ({tkind}); TF32's nominal rate is half of bf16's"})
    dom_i = int(np.argmax(op_ms))
    dom = suite.ops[dom_i]
    achieved = dom[1] / (op_ms[dom_i] / 1e3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(dom[0])
        except Exception:
            traffic = None
    cpu = None
    if world == 1 and not args.no_cpu_baseline and not args.only:
        kind, cores, cops, _ = cpu_suite_sample(1.0)
        dt, by, el, _ = time_cpu(cops, reps=1)
        cpu = {"value": round(by / dt / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": kind,
               "sample": "one pass: cfg1-cfg4 at BASELINE shapes except Snake on 64 of 8192 rows; cfg5 f32 ops on 2^24 elements"}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (Philox4x32-10 seed 0 on the device, BASELINE shapes and distributions)",
        "config": {"workload": "vox-hotpath-suite", "sweep_elems_per_gpu": args.sweep_elems,
                   "bytes_per_step_per_gpu": suite.bytes_per_step, "elements_per_step_per_gpu": suite.elems_per_step,
                   "parallelism": f"row shards x{world}, NCCL all-reduce of 840 f64 slots for the global sum",
                   "scale_cfg1_cfg4": args.scale,
                   "l2": "no flush: the step streams ~%.1f GB per GPU (> 126 MB L2), so every input is evicted by the other ops' "
                         "traffic between its uses" % (suite.bytes_per_step / 1e9)},
        "elements_per_s": round(suite.elems_per_step * world / step_s, 1),
        "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 3), "traffic": traffic, "peak_source": peak_kind},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": suite.launches_per_step * args.steps,
        "clocks": clk.summary(), "ops": ops,
    }
    print(json.dumps(line), flush=True)


def run_e2e(suite, torch, dist, world, steps) -> dict:
    """The suite through the public API with pinned host buffers. Every step copies each op's inputs host->device
    (before their first reader), runs the ops, and copies each op's outputs device->host (after their last writer).
    Copies in, kernels and copies out run on three streams so PCIe traffic in both directions overlaps the kernels
    of neighbouring ops; the ops run in the order of Suite.e2e_order. Returns the same metric as the device-resident
    run (algorithmic GB/s)."""
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    order = suite.e2e_order()
    copy_in, copy_out = suite.copy_plan(order)
    tensors = [t for c in copy_in for t in c] + [t for c in copy_out for t in c]
    pin = {id(t): torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in tensors}
    for c in copy_in:
        for t in c:
            pin[id(t)].copy_(t)
    h2d = sum(t.numel() * t.element_size() for c in copy_in for t in c)
    d2h = sum(t.numel() * t.element_size() for c in copy_out for t in c)
    ev = lambda: torch.cuda.Event()  # noqa: E731

    def one():
        start = ev()
        start.record(comp)
        s_in.wait_event(start)  # inputs of this step are overwritten only after the previous step's kernels
        s_out.wait_event(start)
        for pos, i in enumerate(order):
            e_in = ev()
            with torch.cuda.stream(s_in):
                for t in copy_in[pos]:
                    t.copy_(pin[id(t)], non_blocking=True)
                e_in.record(s_in)
            comp.wait_event(e_in)
            suite.ops[i][3]()
            if copy_out[pos]:
                e_c = ev()
                e_c.record(comp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(e_c)
                    for t in copy_out[pos]:
                        pin[id(t)].copy_(t, non_blocking=True)
        done = ev()
        done.record(s_out)
        comp.wait_event(done)  # outputs are copied out before the next step's kernels overwrite them

    one()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(comp)
    for _ in range(steps):
        one()
    b.record(comp)
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    s = float(ms[0]) / 1e3 / steps
    return {"value": round(suite.bytes_per_step * world / s / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps,
            "overlap": "copy-in / kernels / copy-out on three streams, op groups in Johnson order"}


def run_sweep(args) -> None:
    """BASELINE cfg5 across sizes: for every total size 2^lo .. 2^hi elements (split over the ranks by rows of 4096),
    add / mul / GELU / row sum / max / L2 and the global sum in f32 and bf16, each op timed alone with CUDA events
    (max over ranks). One JSON line on rank 0 with GB/s and elements/s per op and size."""
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    import vox_b200 as vox
    from vox_b200.shard import shard_rows

    peak, _ = peaks()
    results = []
    for lg in range(args.sweep_lo, args.sweep_hi + 1):
        total = 1 << lg
        R = total // 4096
        r0, rows = shard_rows(R, world, rank)
        for dt, tag, es in ((torch.float32, "f32", 4), (torch.bfloat16, "bf16", 2)):
            dev = torch.device("cuda", local)
            a = vox.fill_philox(torch.empty(rows, 4096, dtype=dt, device=dev), 1, 0, 1, seed=0, stream_id=16, counter0=r0 * 4096)
            b = vox.fill_philox(torch.empty(rows, 4096, dtype=dt, device=dev), 1, 0, 1, seed=0, stream_id=18, counter0=r0 * 4096)
            y, rr = torch.empty_like(a), torch.empty(rows, device=dev)
            slots, scratch, gout = (torch.empty(840, dtype=torch.float64, device=dev), torch.empty(max(rows, 1), device=dev),
                                    torch.empty(1, dtype=torch.float64, device=dev))
            n = rows * 4096

            def gsum():
                vox.global_sum_partials(a, r0, R, slots=slots, scratch=scratch)
                if world > 1:
                    dist.all_reduce(slots)
                vox.global_sum_finish(slots, out=gout)

            ops = [("add", 3 * es, lambda: vox.add(a, b, out=y)), ("mul", 3 * es, lambda: vox.mul(a, b, out=y)),
                   ("gelu", 2 * es, lambda: vox.gelu(a, vox.GELU_ERF, out=y)),
                   ("rowsum", es, lambda: vox.row_reduce(a, vox.REDUCE_SUM, out=rr)),
                   ("rowmax", es, lambda: vox.row_reduce(a, vox.REDUCE_MAX, out=rr)),
                   ("rowl2", es, lambda: vox.row_reduce(a, vox.REDUCE_L2, out=rr))]
            if tag == "f32":
                ops.append(("global_sum", es, gsum))
            for name, bpe, fn in ops:
                iters = max(5, min(200, int(2e-3 / max(n * bpe / (peak * 1e9), 1e-7))))
                for _ in range(3):
                    fn()
                torch.cuda.synchronize()
                if world > 1:
                    dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                t = torch.tensor([e0.elapsed_time(e1) / iters], dtype=torch.float64, device=dev)
                if world > 1:
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                sec = float(t) / 1e3
                nbytes = total * bpe + (R * 4 if name.startswith("row") or name == "global_sum" else 0)
                results.append({"elements": total, "log2": lg, "dtype": tag, "op": name, "us": round(sec * 1e6, 2),
                                "gb_s": round(nbytes / sec / 1e9, 1), "frac_of_peak": round(nbytes / sec / 1e9 / peak, 3),
                                "elements_per_s": round(total / sec, 1)})
            del a, b, y, rr
            torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"metric": METRIC, "mode": "sweep", "n_gpus": world, "unit": "GB/s", "peak": peak,
                          "config": {"workload": "BASELINE cfg5 sweep", "sizes": f"2^{args.sweep_lo}..2^{args.sweep_hi} elements in total",
                                     "rows": 4096, "scaling": "strong within a size (total elements fixed)"},
                          "results": results}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--sweep-elems", type=int, default=1 << 27, help="per-GPU elements of each cfg5 tensor (multiple of 4096)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", default=None, help="regex: run only the matching ops (profiling one kernel)")
    ap.add_argument("--sweep", action="store_true", help="BASELINE cfg5 size sweep instead of the suite")
    ap.add_argument("--scale", type=int, default=1, help="multiply the rows/heads/batches of cfg1-cfg4 (1 = BASELINE shapes)")
    ap.add_argument("--sweep-lo", type=int, default=20)
    ap.add_argument("--sweep-hi", type=int, default=32)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.sweep:
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
