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

def make_comm(vox, torch, dist, rank: int, world: int):
    """The library's communicator over the ranks (None on one GPU): rank 0 draws the id, torch.distributed carries it."""
    if world <= 1:
        return None
    uid = torch.zeros(vox.Comm.ID_BYTES, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(vox.Comm.unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    return vox.Comm(bytes(uid.cpu().numpy()), world, rank)


class Suite:
    """Device buffers and the per-op launch list of one step. `ops` entries: (name, bytes, elements, fn).

    `only` (a regex) keeps the matching ops and allocates only their buffers (profiling of one kernel)."""

    def __init__(self, vox, torch, rank: int, world: int, sweep_elems: int, dist=None, only: str | None = None, scale: int = 1, comm=None):
        import re

        self.vox, self.t, self.rank, self.world, self.dist = vox, torch, rank, world, dist
        self.comm = comm
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
        """One library call: this shard's slot partials, the all-reduce of the 840 slots over the library's own NCCL
        communicator (world > 1), the fixed-order fold."""
        self.vox.global_sum_comm(self.gsum_x, self.g_row0, self.g_rows_total, self.comm, slots=self.slots, scratch=self.gscratch,
                                 out=self.gout)

    def step(self, events=None):
        for i, (_, _, _, fn) in enumerate(self.ops):
            if events is not None:
                events[i][0].record()
            fn()
            if events is not None:
                events[i][1].record()


# ---------------------------------------------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU during the timed region, read (never set) through
    NVML in a thread every 2 ms, so that even a timed region of a few tens of ms holds samples; nvidia-smi at 200 ms
    (`-lms 200`) where NVML is not importable. Median SM MHz under load, the maximum SM MHz, the reasons seen."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h): SW power cap, HW slowdown, SW thermal, HW thermal
    BITS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40))

    def __init__(self, gpu_index: int):
        self.idx, self.proc, self.lines = gpu_index, None, []
        self.nv, self.h, self.samples, self.mask, self.max_mhz, self.stop = None, None, [], 0, None, threading.Event()

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:  # the device torch sees as this index (CUDA_VISIBLE_DEVICES may renumber)
            uuid = str(torch.cuda.get_device_properties(self.idx).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.idx)

    def __enter__(self):
        try:
            self.nv, self.h = self._nvml_handle()
            self.max_mhz = float(self.nv.nvmlDeviceGetMaxClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            reasons = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or self.nv.nvmlDeviceGetCurrentClocksThrottleReasons

            def poll():
                while not self.stop.is_set():
                    try:
                        self.samples.append(float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)))
                        self.mask |= int(reasons(self.h))
                    except Exception:
                        pass
                    self.stop.wait(0.002)

            self.th = threading.Thread(target=poll, daemon=True)
            self.th.start()
            return self
        except Exception:
            self.nv = None
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
        self.stop.set()
        if self.nv is not None:
            self.th.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self.nv is not None:
            reasons = sorted(nm for nm, bit in self.BITS if self.mask & bit)
            return {"sm_mhz": float(np.median(self.samples)) if self.samples else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml"}
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
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvidia-smi"}


# ---------------------------------------------------------------------------------------------------- CPU reference

def suite_model(sweep_elems: int, scale: int = 1) -> list[tuple[str, int, int]]:
    """(name, algorithmic bytes, elements) of every op of the default suite per GPU, in launch order: the byte model
    both arms report against (each input read once, each output written once, at the stated element types)."""
    K, n = scale, sweep_elems
    m1, H2, B3, R4, B4 = 512 * K, 16 * K, 8 * K, 4096 * K, 16 * K
    rows = n // 4096
    ops = [("cfg1_rmsnorm_f32", 2 * m1 * 1024 * 4 + 1024 * 4, m1 * 1024),
           ("cfg1_swiglu_f32", 3 * m1 * 3072 * 4, m1 * 3072),
           ("cfg2_softmax_causal_f32", H2 * 1024 * 1025 // 2 * 4 + H2 * 1024 * 1024 * 4, H2 * 1024 * 1024),
           ("cfg3_adaln_bf16", 3 * B3 * 2048 * 1024 * 2 + 3 * B3 * 1024 * 2, B3 * 2048 * 1024),
           ("cfg4_dequant_q8_bf16", R4 * 4096 + R4 * 128 * 2 + R4 * 4096 * 2, R4 * 4096),
           ("cfg4_dequant_q4_bf16", R4 * 2048 + R4 * 128 * 2 + R4 * 4096 * 2, R4 * 4096),
           ("cfg4_snake_hift_f32", 2 * B4 * 512 * 24000 * 4 + 512 * 4, B4 * 512 * 24000)]
    for tag, es in (("f32", 4), ("bf16", 2)):
        ops += [(f"cfg5_add_{tag}", 3 * n * es, n), (f"cfg5_mul_{tag}", 3 * n * es, n), (f"cfg5_gelu_{tag}", 2 * n * es, n)]
        ops += [(f"cfg5_{k}_{tag}", n * es + rows * 4, n) for k in ("rowsum", "rowmax", "rowl2")]
        if es == 4:
            ops.append(("cfg5_global_sum_f32", n * 4 + rows * 4, n))
    return ops


def suite_config(sweep_elems: int, scale: int = 1) -> dict:
    """The `config` of the default suite: identical in both arms (the GPU's and the reference CPU's)."""
    model = suite_model(sweep_elems, scale)
    nb = sum(b for _, b, _ in model)
    return {"workload": "vox-hotpath-suite", "ops": [nm for nm, _, _ in model], "sweep_elems_per_gpu": sweep_elems,
            "bytes_per_step_per_gpu": nb, "elements_per_step_per_gpu": sum(e for _, _, e in model), "scale_cfg1_cfg4": scale,
            "l2": "no flush: inputs larger than L2 - each step streams %.1f GB per GPU through a 126 MB L2, so every input "
                  "is evicted by the other ops' traffic between its uses" % (nb / 1e9)}


def cpu_model() -> str:
    try:
        for ln in subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout.splitlines():
            if ln.startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


class CpuSuite:
    """The default suite on the host through dariumi/Vox's own CPU operators (oracle/_ref/libvox_ref.so, compiled
    from the reference sources; the C restatement where that library is absent): the same ops as the GPU suite, at
    the same shapes and element types in memory (bf16 tensors stay bf16, widened and rounded inside the parallel
    loops), on the same Philox4x32-10 inputs, with every output preallocated outside the timed region. Threads: all
    host cores through Vox's own ThreadPool (vox::set_num_threads(0)) with Vox's grains."""

    def __init__(self, sweep_elems: int):
        from oracle.oracle import port, ref

        P, R = port(), ref()
        self.kind = "reference" if R is not None else "port"
        self.cores = R.set_threads(0) if R is not None else 1
        f32, u16 = np.float32, np.uint16
        E = lambda *sh, dt=f32: np.empty(sh, dt)  # noqa: E731
        nrm = lambda sh, sid, m=0.0, sd=1.0: P.fill_into(E(*sh), 1, m, sd, sid=sid)  # noqa: E731
        uni = lambda sh, sid, lo, hi: P.fill_into(E(*sh), 0, lo, hi, sid=sid)  # noqa: E731

        def nrm16(sh, sid, m=0.0, sd=1.0):
            return P.bf16_round_into(nrm(sh, sid, m, sd), E(*sh, dt=u16))

        pt = lambda a: a.ctypes.data  # noqa: E731
        ops = []
        model = {nm: (b, e) for nm, b, e in suite_model(sweep_elems)}

        def add(name, fn):
            ops.append((name, model[name][0], model[name][1], fn))

        # cfg1
        x1, w1, y1 = nrm((512, 1024), 1), nrm((1024,), 2, 1, 0.02), E(512, 1024)
        g1, u1, h1 = nrm((512, 3072), 3), nrm((512, 3072), 4), E(512, 3072)
        # cfg2
        s2, p2 = nrm((16, 1024, 1024), 5, 0, 3), E(16, 1024, 1024)
        # cfg3 (bf16 activations and parameters)
        x3, r3 = nrm16((8, 2048, 1024), 6), nrm16((8, 2048, 1024), 7)
        sh3, sc3, g3 = (nrm16((8, 1024), sid, 0, 0.1) for sid in (8, 9, 10))
        m3, y3 = E(2048, 1024), E(8, 2048, 1024, dt=u16)
        # cfg4: f16 scales widened once to the f32 scales Vox's Mat holds
        s4 = P.f16_to_f32(uni((4096, 128), 13, 0.001, 0.05).astype(np.float16).view(u16))
        q8, q4 = P.fill_into(E(4096, 4096, dt=np.int8), 2, -128, 127, sid=11), P.fill_into(E(4096, 2048, dt=np.uint8), 3, sid=12)
        o8, o4 = E(4096, 4096, dt=u16), E(4096, 4096, dt=u16)
        xs, al, ys = nrm((16, 512, 24000), 14), uni((512,), 15, 0.2, 2.0), E(16, 512, 24000)
        # cfg5
        n, rows = sweep_elems, sweep_elems // 4096
        a5, b5, y5 = nrm((rows, 4096), 16), nrm((rows, 4096), 18), E(rows, 4096)
        a6, b6, y6 = nrm16((rows, 4096), 17), nrm16((rows, 4096), 19), E(rows, 4096, dt=u16)
        rr, slots = E(rows), np.empty(840, np.float64)
        self._keep = [x1, w1, y1, g1, u1, h1, s2, p2, x3, r3, sh3, sc3, g3, m3, y3, s4, q8, q4, o8, o4, xs, al, ys, a5, b5, y5, a6, b6, y6,
                      rr, slots]
        sc2 = float(1.0 / np.sqrt(128.0))
        if R is not None:
            L = R.L
            add("cfg1_rmsnorm_f32", lambda: L.vr_rmsnorm_rows(pt(x1), pt(w1), 512, 1024, 1e-6, pt(y1), 1))
            add("cfg1_swiglu_f32", lambda: L.vr_silu_mul(pt(g1), pt(u1), pt(h1), g1.size))
            add("cfg2_softmax_causal_f32", lambda: L.vr_softmax_rows(pt(s2), pt(p2), 16 * 1024, 1024, sc2, 1024, 0, 0))
            add("cfg3_adaln_bf16", lambda: L.vr_adaln_bf16(pt(x3), pt(sh3), pt(sc3), pt(g3), pt(r3), 8, 2048, 1024, pt(m3), pt(y3)))
            add("cfg4_dequant_q8_bf16", lambda: L.vr_mat_rows_bf16(3, pt(q8), pt(s4), 4096, 4096, pt(o8)))
            add("cfg4_dequant_q4_bf16", lambda: L.vr_mat_rows_bf16(4, pt(q4), pt(s4), 4096, 4096, pt(o4)))
            add("cfg4_snake_hift_f32", lambda: L.vr_snake(pt(xs), pt(al), None, pt(ys), xs.size, 512, 24000, 0))
            add("cfg5_add_f32", lambda: L.vr_add(pt(a5), pt(b5), pt(y5), n))
            add("cfg5_mul_f32", lambda: L.vr_mul(pt(a5), pt(b5), pt(y5), n))
            add("cfg5_gelu_f32", lambda: L.vr_gelu_f32(pt(a5), pt(y5), n))
            for op, nm in ((0, "rowsum"), (1, "rowmax"), (2, "rowl2")):
                add(f"cfg5_{nm}_f32", lambda op=op: L.vr_row_reduce(pt(a5), pt(rr), rows, 4096, op))
            add("cfg5_global_sum_f32", lambda: L.vr_global_sum(pt(a5), rows, 4096, pt(rr), pt(slots)))
            add("cfg5_add_bf16", lambda: L.vr_add_bf16(pt(a6), pt(b6), pt(y6), n))
            add("cfg5_mul_bf16", lambda: L.vr_mul_bf16(pt(a6), pt(b6), pt(y6), n))
            add("cfg5_gelu_bf16", lambda: L.vr_gelu_bf16(pt(a6), pt(y6), n))
            for op, nm in ((0, "rowsum"), (1, "rowmax"), (2, "rowl2")):
                add(f"cfg5_{nm}_bf16", lambda op=op: L.vr_row_reduce_bf16(pt(a6), pt(rr), rows, 4096, op))
        else:  # the single-threaded C restatement (a machine without the reference library); bf16 tensors widened once
            from oracle.oracle import bf16_bits_to_f32 as wide

            Q = P.L
            x3f, r3f, sh3f, sc3f, g3f, y3f = wide(x3), wide(r3), wide(sh3), wide(sc3), wide(g3), E(8, 2048, 1024)
            a6f, b6f, y6f = wide(a6), wide(b6), E(rows, 4096)
            self._keep += [x3f, r3f, sh3f, sc3f, g3f, y3f, a6f, b6f, y6f]
            add("cfg1_rmsnorm_f32", lambda: Q.vo_rmsnorm_rows(pt(x1), pt(w1), 512, 1024, 1e-6, pt(y1)))
            add("cfg1_swiglu_f32", lambda: Q.vo_silu_mul(pt(g1), pt(u1), pt(h1), g1.size))
            add("cfg2_softmax_causal_f32", lambda: Q.vo_softmax_rows(pt(s2), pt(p2), 16 * 1024, 1024, sc2, 1024, 0))
            add("cfg3_adaln_bf16", lambda: Q.vo_adaln(pt(x3f), pt(sh3f), pt(sc3f), pt(g3f), pt(r3f), 8, 2048, 1024, 1e-6, pt(y3f)))
            add("cfg4_dequant_q8_bf16", lambda: Q.vo_dequant_q8(pt(q8), pt(s4), 4096, 4096, pt(y3f)))
            add("cfg4_dequant_q4_bf16", lambda: Q.vo_dequant_q4(pt(q4), pt(s4), 4096, 4096, pt(y3f)))
            add("cfg4_snake_hift_f32", lambda: Q.vo_snake(pt(xs), pt(al), None, pt(ys), xs.size, 512, 24000, 0))
            for tag, (a, b, y) in (("f32", (a5, b5, y5)), ("bf16", (a6f, b6f, y6f))):
                add(f"cfg5_add_{tag}", lambda a=a, b=b, y=y: Q.vo_add(pt(a), pt(b), pt(y), n))
                add(f"cfg5_mul_{tag}", lambda a=a, b=b, y=y: Q.vo_mul(pt(a), pt(b), pt(y), n))
                add(f"cfg5_gelu_{tag}", lambda a=a, y=y: Q.vo_gelu_erf(pt(a), pt(y), n))
                for op, nm in ((0, "rowsum"), (1, "rowmax"), (2, "rowl2")):
                    add(f"cfg5_{nm}_{tag}", lambda op=op, a=a: Q.vo_row_reduce_f64(pt(a), pt(rr), rows, 4096, op))
            add("cfg5_global_sum_f32", lambda: Q.vo_row_reduce_f64(pt(a5), pt(rr), rows, 4096, 0))
        order = [nm for nm, _, _ in suite_model(sweep_elems)]
        ops.sort(key=lambda o: order.index(o[0]))
        self.ops = ops
        self.bytes_per_step = sum(o[1] for o in ops)
        self.elems_per_step = sum(o[2] for o in ops)

    def time(self, steps: int, warmup: int, budget_s: float = 240.0) -> tuple[float, int, int, dict, str]:
        """Times `steps` steps after `warmup` untimed ones. A step is one pass over every op when (steps + warmup)
        passes fit in `budget_s`; otherwise each step runs the next op of the suite in turn (a bounded sample whose
        aggregate over the steps weights the ops as a full pass does). Returns (seconds, bytes, elements, per-op
        seconds, sample description)."""
        t0 = time.perf_counter()
        for *_, fn in self.ops:
            fn()
        one = time.perf_counter() - t0
        full = (steps + max(warmup - 1, 0)) * one <= budget_s
        plan = [list(range(len(self.ops))) for _ in range(steps)] if full else \
            [[k % len(self.ops)] for k in range(steps)]
        for _ in range(max(warmup - 1, 0)):
            for i in (range(len(self.ops)) if full else [0]):
                self.ops[i][3]()
        per, runs, nbytes, nel = {}, {}, 0, 0
        t0 = time.perf_counter()
        for idx in plan:
            for i in idx:
                nm, by, el, fn = self.ops[i]
                s = time.perf_counter()
                fn()
                per[nm] = per.get(nm, 0.0) + time.perf_counter() - s
                runs[nm] = runs.get(nm, 0) + 1
                nbytes += by
                nel += el
        dt = time.perf_counter() - t0
        sample = ("every step one full pass of the suite: the GPU arm's ops, shapes and element types" if full else
                  "every step the next op of the suite in turn (a full pass per step would exceed %.0f s)" % budget_s)
        return dt, nbytes, nel, per, runs, sample

    def op_table(self, per: dict, runs: dict) -> dict:
        """Per-op GB/s and milliseconds of a timed run."""
        return {nm: {"gb_s": round(by * runs[nm] / per[nm] / 1e9, 3), "ms": round(per[nm] / runs[nm] * 1e3, 3)}
                for nm, by, _, _ in self.ops if nm in per}


def run_reference(args) -> None:
    """The reference arm: dariumi/Vox's own CPU operators on the host cores over the GPU arm's suite (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cs = CpuSuite(args.sweep_elems)
    dt, by, el, per, runs, sample = cs.time(args.steps, args.warmup)
    value = by / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (Philox4x32-10 seed 0, BASELINE shapes and distributions; the GPU arm's inputs)",
        "config": suite_config(args.sweep_elems),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cs.cores, "kind": cs.kind, "cpu_model": cpu_model(),
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "elements_per_s": round(el / dt, 1),
        "ops": cs.op_table(per, runs),
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

    comm = make_comm(vox, torch, dist, rank, world)
    suite = Suite(vox, torch, rank, world, args.sweep_elems, dist if world > 1 else None, only=args.only, scale=args.scale, comm=comm)
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
        torch.cuda.nvtx.range_push("timed")  # profilers can select the timed steps' kernels by this range
        t0.record()
        for k in range(args.steps):
            suite.step()
        t1.record()
        torch.cuda.nvtx.range_pop()
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
        torch.cuda.synchronize()
        dist.barrier()
        if comm is not None:
            comm.close()
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
        cs = CpuSuite(args.sweep_elems)
        dt, by, el, per, runs, _ = cs.time(1, 1)
        cpu = {"value": round(by / dt / 1e9, 3), "unit": "GB/s", "cores": cs.cores, "kind": cs.kind, "cpu_model": cpu_model(),
               "sample": "one full pass of the suite after one untimed pass: the GPU arm's ops, shapes and element types",
               "ops": cs.op_table(per, runs)}
        del cs
    if args.only is None and args.scale == 1:
        config = suite_config(args.sweep_elems)  # the default suite: the reference arm's config
        assert config["bytes_per_step_per_gpu"] == suite.bytes_per_step and config["ops"] == [o[0] for o in suite.ops]
    else:
        config = {"workload": "vox-hotpath-suite" + (f" (ops matching {args.only!r})" if args.only else ""),
                  "ops": [o[0] for o in suite.ops], "sweep_elems_per_gpu": args.sweep_elems, "bytes_per_step_per_gpu": suite.bytes_per_step,
                  "elements_per_step_per_gpu": suite.elems_per_step, "scale_cfg1_cfg4": args.scale}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (Philox4x32-10 seed 0 on the device, BASELINE shapes and distributions)",
        "config": config,
        "parallelism": f"row shards x{world}, NCCL all-reduce of 840 f64 slots for the global sum",
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
    comm = make_comm(vox, torch, dist, rank, world)
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
                vox.global_sum_comm(a, r0, R, comm, slots=slots, scratch=scratch, out=gout)

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
        torch.cuda.synchronize()
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"metric": METRIC, "mode": "sweep", "n_gpus": world, "unit": "GB/s", "peak": peak,
                          "config": {"workload": "BASELINE cfg5 sweep", "sizes": f"2^{args.sweep_lo}..2^{args.sweep_hi} elements in total",
                                     "rows": 4096, "scaling": "strong within a size (total elements fixed)"},
                          "results": results}), flush=True)


def run_copy_roofline(args) -> None:
    """Size-matched copy roofline of the small BASELINE configs: for each op, the op alone and a plain device copy of
    the same traffic (a torch copy_ of bytes/2: reads bytes/2, writes bytes/2), both timed the same way - CUDA events
    around back-to-back launches that rotate over enough buffer sets that the sets total at least 3x the L2 size (so
    every launch reads HBM) - on one GPU. frac_of_copy = copy time / op time: the fraction of the bandwidth that this
    size of transfer attains at all. One JSON line."""
    import torch

    torch.cuda.set_device(0)
    import vox_b200 as vox

    peak, _ = peaks()
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    names = ["cfg1_rmsnorm_f32", "cfg1_swiglu_f32", "cfg2_softmax_causal_f32", "cfg3_adaln_bf16", "cfg4_dequant_q8_bf16",
             "cfg4_dequant_q4_bf16", "cfg4_snake_hift_f32"]
    if args.only:
        import re

        names = [nm for nm in names if re.search(args.only, nm)]
    res = {}

    def timed(fns, reps):
        for f in fns:
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # a spin kernel holds the GPU while the host enqueues every launch, so no host launch cost is timed
        torch.cuda._sleep(int(min(max(0.03 * reps, 5.0), 2000.0) * 2.0e6))
        e0.record()
        for k in range(reps):
            fns[k % len(fns)]()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3  # us

    for nm in names:
        nb = dict((o[0], o[1]) for o in suite_model(args.sweep_elems))[nm]
        sets = max(2, -(-3 * l2 // nb))
        suites = [Suite(vox, torch, 0, 1, args.sweep_elems, only=f"^{nm}$") for _ in range(sets)]
        fns = [su.ops[0][3] for su in suites]
        reps = max(3 * sets, 60)
        op_us = min(timed(fns, reps) for _ in range(3))
        del suites, fns
        torch.cuda.empty_cache()
        half = nb // 2
        bufs = [(torch.empty(half, dtype=torch.uint8, device="cuda"), torch.empty(half, dtype=torch.uint8, device="cuda"))
                for _ in range(sets)]
        cps = [lambda s=s_, d=d_: d.copy_(s) for s_, d_ in bufs]
        cp_us = min(timed(cps, reps) for _ in range(3))
        del bufs, cps
        torch.cuda.empty_cache()
        res[nm] = {"bytes": nb, "op_us": round(op_us, 2), "copy_us": round(cp_us, 2), "op_gb_s": round(nb / op_us / 1e3, 1),
                   "copy_gb_s": round(nb / cp_us / 1e3, 1), "frac_of_copy": round(cp_us / op_us, 3),
                   "frac_of_peak": round(nb / op_us / 1e3 / peak, 3), "copy_frac_of_peak": round(nb / cp_us / 1e3 / peak, 3),
                   "buffer_sets": sets}
    print(json.dumps({"metric": METRIC, "mode": "copy-roofline", "unit": "GB/s", "peak": peak, "l2_bytes": l2,
                      "config": {"workload": "BASELINE cfg1-cfg4 ops alone against a device copy of the same bytes"},
                      "results": res}), flush=True)


def run_gemv_sweep(args) -> None:
    """The quantized decode GEMV (one activation row, [rows][4096] weights with f16 scales) over a range of matrix
    heights, on one GPU, each size timed three ways: an event pair around every launch (as the suite's per-op numbers),
    back-to-back launches (the mean; consecutive launches may overlap their set-up), and a plain device copy of the
    same bytes (a torch copy_ of bytes/2, back to back). Every timing rotates over enough matrices that they total at
    least 3x the L2 size, so every launch reads HBM. A least-squares line through the two largest sizes splits the
    per-launch time into a fixed part (us) and a marginal rate (GB/s). One JSON line."""
    import torch

    torch.cuda.set_device(0)
    import vox_b200 as vox

    peak, _ = peaks()
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    cols, res = 4096, {}
    for qt in ("q8", "q4"):
        fn = vox.gemv_q8 if qt == "q8" else vox.gemv_q4
        pts = []
        for rows in (3072, 6144, 12288, 24576, 49152):
            wb = rows * cols if qt == "q8" else rows * cols // 2
            nb = wb + rows * (cols // 32) * 2 + cols * 4 + rows * 4
            sets = max(2, -(-3 * l2 // nb))
            gen = torch.Generator(device="cuda").manual_seed(rows)
            if qt == "q8":
                mats = [torch.randint(-128, 128, (rows, cols), dtype=torch.int8, device="cuda", generator=gen) for _ in range(sets)]
            else:
                mats = [torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device="cuda", generator=gen) for _ in range(sets)]
            scs = [(torch.rand(rows, cols // 32, device="cuda", generator=gen) * 0.05 + 0.001).half() for _ in range(sets)]
            x = torch.randn(1, cols, device="cuda", generator=gen)
            y = torch.empty(1, rows, device="cuda")
            calls = [lambda i=i: fn(mats[i], scs[i], x, out=y) for i in range(sets)]
            reps = max(3 * sets, 60)
            for c in calls:
                c()
            torch.cuda.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            torch.cuda._sleep(int(min(max(0.06 * reps, 5.0), 2000.0) * 2.0e6))  # the host enqueues while the GPU spins
            for k in range(reps):
                ev[k][0].record()
                calls[k % sets]()
                ev[k][1].record()
            torch.cuda.synchronize()
            per_launch = float(np.mean([a.elapsed_time(b) for a, b in ev])) * 1e3

            def b2b(fns):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(int(min(max(0.03 * reps, 5.0), 2000.0) * 2.0e6))
                e0.record()
                for k in range(reps):
                    fns[k % len(fns)]()
                e1.record()
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) / reps * 1e3

            back = min(b2b(calls) for _ in range(3))
            del mats, scs, calls
            torch.cuda.empty_cache()
            bufs = [(torch.empty(nb // 2, dtype=torch.uint8, device="cuda"), torch.empty(nb // 2, dtype=torch.uint8, device="cuda"))
                    for _ in range(sets)]
            cps = [lambda s=s_, d=d_: d.copy_(s) for s_, d_ in bufs]
            for c in cps:
                c()
            cp = min(b2b(cps) for _ in range(3))
            del bufs, cps
            torch.cuda.empty_cache()
            pts.append((nb, per_launch))
            res[f"{qt}_{rows}x{cols}"] = {"bytes": nb, "per_launch_us": round(per_launch, 2), "back_to_back_us": round(back, 2),
                                          "copy_us": round(cp, 2), "per_launch_frac_of_peak": round(nb / per_launch / 1e3 / peak, 3),
                                          "back_to_back_frac_of_peak": round(nb / back / 1e3 / peak, 3),
                                          "copy_frac_of_peak": round(nb / cp / 1e3 / peak, 3), "frac_of_copy": round(cp / back, 3)}
        (b1, t1), (b2, t2) = pts[-2], pts[-1]
        slope = (t2 - t1) / (b2 - b1)  # us per byte
        res[f"{qt}_fit"] = {"fixed_us": round(t1 - slope * b1, 2), "marginal_gb_s": round(1.0 / slope / 1e3, 1),
                            "marginal_frac_of_peak": round(1.0 / slope / 1e3 / peak, 3)}
    print(json.dumps({"metric": METRIC, "mode": "gemv-sweep", "unit": "GB/s", "peak": peak, "l2_bytes": l2,
                      "config": {"workload": "quantized decode GEMV, 1 activation row, [rows][4096] with f16 scales"},
                      "results": res}), flush=True)


def run_gemm(args) -> None:
    """The tcgen05 GEMM (vox_cuda_gemm_bf16) alone on the F5-base projections, a prefill-shaped case and a large square
    case, against torch's bf16 matmul (cuBLAS) on the same operands: CUDA events around back-to-back launches, one
    GPU. One JSON line."""
    import torch

    torch.cuda.set_device(0)
    import vox_b200 as vox

    tpk, tkind = tensor_peak()
    shapes = [("f5_qkv", 2048, 3072, 1024), ("f5_o", 2048, 1024, 1024), ("f5_ff1", 2048, 2048, 1024), ("f5_ff2", 2048, 1024, 2048),
              ("prefill_up", 512, 12288, 4096), ("square_8192", 8192, 8192, 8192)]
    if args.gemm_shape:  # one shape only (profiling a single kernel)
        m, n, k = (int(v) for v in args.gemm_shape.lower().split("x"))
        shapes = [(f"gemm_{m}x{n}x{k}", m, n, k)]
    if args.gemm_quant:  # the quantized prefill GEMM only
        shapes = []
    res = {}
    g = torch.Generator(device="cuda").manual_seed(0)
    reps = 40

    def t(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(min(max(0.03 * reps, 5.0), 2000.0) * 2.0e6))  # the host enqueues while the GPU spins
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3

    for nm, m, n, k in shapes:
        x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
        y = torch.empty(m, n, device="cuda")
        yb = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        fl = 2 * m * n * k
        reps = max(5, min(200, int(2e-3 / (fl / 1.2e15))))

        ours = min(t(lambda: vox.gemm_bf16(x, w, out=y)) for _ in range(3))
        ours_b = min(t(lambda: vox.gemm_bf16(x, w, out_dtype=torch.bfloat16, out=yb)) for _ in range(3))
        ref = min(t(lambda: torch.matmul(x, w.t(), out=yb)) for _ in range(3))
        # weights rotated over copies totalling more than twice the L2, so each launch reads its W from HBM (as the
        # layers of a model do)
        ncopy = max(2, -(-300_000_000 // (n * k * 2)))
        ws = [w.clone() for _ in range(ncopy)] if ncopy <= 64 else None
        cold = cold_ref = None
        if ws is not None:
            ctr = [0]

            def rot(fn):
                def f():
                    ctr[0] += 1
                    fn(ws[ctr[0] % ncopy])
                return f

            cold = min(t(rot(lambda wi: vox.gemm_bf16(x, wi, out_dtype=torch.bfloat16, out=yb))) for _ in range(3))
            cold_ref = min(t(rot(lambda wi: torch.matmul(x, wi.t(), out=yb))) for _ in range(3))
            del ws
        res[nm] = {"m": m, "n": n, "k": k, "us_f32_out": round(ours, 2), "us_bf16_out": round(ours_b, 2), "cublas_bf16_us": round(ref, 2),
                   "tflops": round(fl / ours_b / 1e6, 1), "frac_of_tensor_peak": round(fl / ours_b / 1e6 / tpk, 3),
                   "cublas_tflops": round(fl / ref / 1e6, 1),
                   "cold_w_us": None if cold is None else round(cold, 2), "cold_w_cublas_us": None if cold_ref is None else round(cold_ref, 2)}
        del x, w, y, yb
    # the quantized prefill GEMM (Q8 / Q4 weights [n][4096] with f16 scales, 512 f32 activation rows), weights rotated
    # over enough copies that they stream from HBM; `us` is the default form (two passes from 256 rows of x), also
    # timed in one pass (VOX_CUDA_GEMMQ_TWOPASS=0) and in one pass on whole tiles (VOX_CUDA_GEMMQ_SPLIT=0); the
    # library reads both at every call
    for m, n, k in ((512, 12288, 4096), (512, 4096, 4096)):
        x = torch.randn(m, k, device="cuda", generator=g)
        y = torch.empty(m, n, device="cuda")
        fl = 2 * m * n * k
        for qt in ("q8", "q4"):
            mats = [vox.fill_philox(torch.empty(n, k if qt == "q8" else k // 2, dtype=torch.int8 if qt == "q8" else torch.uint8, device="cuda"),
                                    2 if qt == "q8" else 3, -128, 127, seed=0, stream_id=70 + i) for i in range(4)]
            scs = [vox.fill_philox(torch.empty(n, k // 32, device="cuda"), 0, 0.001, 0.05, seed=0, stream_id=80 + i).half() for i in range(4)]
            fn = vox.gemm_q8 if qt == "q8" else vox.gemm_q4
            ctr = [0]

            def call(fn=fn, mats=mats, scs=scs, ctr=ctr):
                i = ctr[0] % 4
                ctr[0] += 1
                fn(mats[i], scs[i], x, out=y)

            reps = 40
            us = min(t(call) for _ in range(3))
            os.environ["VOX_CUDA_GEMMQ_TWOPASS"] = "0"
            us_one = min(t(call) for _ in range(3))
            os.environ["VOX_CUDA_GEMMQ_SPLIT"] = "0"
            us_whole = min(t(call) for _ in range(3))
            del os.environ["VOX_CUDA_GEMMQ_SPLIT"], os.environ["VOX_CUDA_GEMMQ_TWOPASS"]
            res[f"prefill_{qt}" + ("" if n == 12288 else f"_{m}x{n}x{k}")] = {
                "m": m, "n": n, "k": k, "us": round(us, 2), "tflops": round(fl / us / 1e6, 1), "frac_of_tensor_peak": round(fl / us / 1e6 / tpk, 3),
                "weight_gb_s": round((n * k * (1 if qt == "q8" else 0.5) + n * k // 32 * 2) / us / 1e3, 1), "us_one_pass": round(us_one, 2), "us_one_pass_whole_tiles": round(us_whole, 2)}
            del mats, scs
    print(json.dumps({"metric": METRIC, "mode": "gemm", "unit": "TFLOP/s", "tensor_peak": f"{tpk} bf16 sustained ({tkind})",
                      "config": {"workload": "tcgen05 bf16 GEMM vs cuBLAS, F5-base and prefill shapes"}, "results": res}), flush=True)


def run_probe(args) -> None:
    """Each operator kernel that the suite does not time (LayerNorm plain and modulate, bias-add, gated add, fused
    SwiGLU, SnakeBeta and Kokoro Snake, mul f32 / bf16, add bf16, row max and L2, the global sum's slot partials and
    fold, the Philox fill) on [rows][1024] tensors (default 131072 rows: 512 MB a f32 tensor, four times L2, so no L2
    flush is needed): `--probe-reps` warm-up launches, then `--probe-reps` launches timed back to back with CUDA events
    behind a spin kernel (no host launch gaps), mean per launch; one JSON line. With `--probe-reps 1` every kernel
    launches once after the input fills: the form an ncu launch list or section capture of all of them takes."""
    import torch

    torch.cuda.set_device(0)
    import vox_b200 as vox

    peak, _ = peaks()
    dev = torch.device("cuda", 0)
    f32, bf16 = torch.float32, torch.bfloat16
    fill = lambda t, d=1, a=0.0, b=1.0, sid=0: vox.fill_philox(t, d, a, b, seed=0, stream_id=sid)  # noqa: E731
    R, D = args.probe_rows, 1024
    x = fill(torch.empty(R, D, device=dev), sid=90)
    xb = fill(torch.empty(R, D, device=dev, dtype=bf16), sid=91)
    y, yb = torch.empty_like(x), torch.empty_like(xb)
    w, b = fill(torch.empty(D, device=dev), 1, 1, 0.1, 92), fill(torch.empty(D, device=dev), 1, 0, 0.1, 93)
    B, T = 8, R // 8
    g = fill(torch.empty(B, D, device=dev), 1, 0, 0.1, 94)
    gu = fill(torch.empty(R // 2, 2 * D, device=dev), sid=95)
    hu = torch.empty(R // 2, D, device=dev)
    C, Tc = 512, R * D // (16 * 512)
    xs = fill(torch.empty(16, C, Tc, device=dev), sid=96)
    al = fill(torch.empty(C, device=dev), 0, 0.2, 2.0, 97)
    be = fill(torch.empty(C, device=dev), 0, 0.5, 1.5, 98)
    ys = torch.empty_like(xs)
    rr = torch.empty(R, device=dev)
    slots, sc, gout = torch.empty(840, dtype=torch.float64, device=dev), torch.empty(R, device=dev), torch.empty(1, dtype=torch.float64, device=dev)
    nb = R * D * 4
    ops = [
        ("layernorm_f32", 2 * nb, lambda: vox.layernorm(x, w, b, 1e-5, out=y)),
        ("layernorm_modulate_f32", 2 * nb, lambda: vox.layernorm(x, w, b, 1e-6, modulate=True, out=y)),
        ("bias_add_f32", 2 * nb, lambda: vox.bias_add(y, b)),
        ("gated_add_f32", 3 * nb, lambda: vox.gated_add(y.view(B, T, D), g, x.view(B, T, D))),
        ("swiglu_fused_f32", 3 * nb // 2, lambda: vox.swiglu_fused(gu, out=hu)),
        ("snake_beta_f32", 2 * nb, lambda: vox.snake(xs, al, vox.SNAKE_BETA, beta=be, out=ys)),
        ("snake_kokoro_f32", 2 * nb, lambda: vox.snake(xs, al, vox.SNAKE_KOKORO, out=ys)),
        ("mul_f32", 3 * nb, lambda: vox.mul(x, y, out=y)),
        ("mul_bf16", 3 * nb // 2, lambda: vox.mul(xb, yb, out=yb)),
        ("add_bf16", 3 * nb // 2, lambda: vox.add(xb, yb, out=yb)),
        ("rowmax_f32", nb + R * 4, lambda: vox.row_reduce(x, vox.REDUCE_MAX, out=rr)),
        ("rowl2_bf16", nb // 2 + R * 4, lambda: vox.row_reduce(xb, vox.REDUCE_L2, out=rr)),
        ("global_sum_partials_f32", nb + R * 4, lambda: vox.global_sum_partials(x, 0, R, slots=slots, scratch=sc)),
        ("global_sum_finish", 840 * 8, lambda: vox.global_sum_finish(slots, out=gout)),
        ("fill_philox_normal_f32", nb, lambda: fill(y, sid=99)),
    ]
    reps = max(1, args.probe_reps)
    torch.cuda.synchronize()
    res = {}
    for nm, by, fn in ops:
        if reps > 1:
            for _ in range(reps):
                fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000 if reps > 1 else 1000)  # holds the stream while the host enqueues the timed launches
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        res[nm] = {"us": round(us, 2), "bytes": by, "gb_s": round(by / us / 1e3, 1), "frac_of_peak": round(by / us / 1e3 / peak, 3)}
    print(json.dumps({"metric": METRIC, "mode": "probe", "unit": "GB/s", "peak": peak,
                      "config": {"workload": f"each kernel outside the suite on [{R}][{D}] tensors, mean of {reps} back-to-back launches"},
                      "results": res}), flush=True)


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
    ap.add_argument("--copy-roofline", action="store_true", help="cfg1-cfg4 ops against a size-matched device copy")
    ap.add_argument("--gemv-sweep", action="store_true", help="the decode GEMV over matrix heights, against a same-bytes copy")
    ap.add_argument("--gemm", action="store_true", help="the tcgen05 GEMM alone against cuBLAS")
    ap.add_argument("--probe", action="store_true", help="one launch of each kernel outside the suite (profiling)")
    ap.add_argument("--gemm-shape", default=None, help="--gemm: one MxNxK shape only")
    ap.add_argument("--gemm-quant", action="store_true", help="--gemm: the quantized prefill GEMM only")
    ap.add_argument("--probe-rows", type=int, default=131072, help="--probe: rows of 1024 elements a tensor")
    ap.add_argument("--probe-reps", type=int, default=20, help="--probe: warm-up and timed launches of each kernel")
    ap.add_argument("--sweep-lo", type=int, default=20)
    ap.add_argument("--sweep-hi", type=int, default=32)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.sweep:
        run_sweep(args)
    elif args.copy_roofline:
        run_copy_roofline(args)
    elif args.gemv_sweep:
        run_gemv_sweep(args)
    elif args.gemm:
        run_gemm(args)
    elif args.probe:
        run_probe(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
