"""GPU tests of the .tmod upload (vox_cuda_tmod_upload, vox_cuda_tmod_upload_dequant): the golden file written by the
reference's tmod_write lands on the device byte for byte, its Q8/Q4 matrices dequantise bit-exactly to the
reference's mat_row output (f32) and to its bf16 rounding, and a file larger than the staging ring (several 16 MB
chunks, a partial last one) arrives intact."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from test_gpu_parity import bf16r, host

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden" / "tiny.tmod"


def test_upload_golden_blobs(vox, golden):
    g = golden["tmod"]
    with vox.Tmod(GOLD) as t:
        names = t.names()
        outs = t.upload(names)
        torch.cuda.synchronize()
        for n, o in zip(names, outs):
            assert o.cpu().contiguous().view(torch.uint8).numpy().tobytes() == t.host_bytes(n), n
        np.testing.assert_array_equal(outs[names.index("layer.w")].cpu().numpy(), g["q8"])


def test_upload_dequant_bitexact(vox, golden):
    g = golden["tmod"]
    with vox.Tmod(GOLD) as t:
        for name, want in (("layer.w", g["q8_deq"]), ("layer.u", g["q4_deq"])):
            y = host(t.upload_dequant(name, torch.float32))
            np.testing.assert_array_equal(y.view(np.uint32), want.astype(np.float32).view(np.uint32))
            yb = host(t.upload_dequant(name, torch.bfloat16))
            np.testing.assert_array_equal(yb.view(np.uint32), bf16r(want).view(np.uint32))


def test_upload_large_file_through_the_ring(vox, tmp_path):
    from vox_b200.tmodfile import write_tmod

    rng = np.random.default_rng(7)
    big = rng.integers(0, 256, 40 * (1 << 20) + 4096 + 48, dtype=np.uint8)  # 40 MB + a bit: 3 chunks, partial last
    small = rng.integers(0, 256, 1000, dtype=np.uint8)
    p = tmp_path / "big.tmod"
    write_tmod(p, {"family": "big"}, {"big": ("U8", (big.size,), big.tobytes()), "small": ("U8", (small.size,), small.tobytes())})
    with vox.Tmod(p) as t:
        for _ in range(2):  # the second pass reuses the staging ring (events gate the reuse)
            ob, os_ = t.upload(["big", "small"])
            torch.cuda.synchronize()
            assert torch.equal(ob, torch.from_numpy(big).cuda())
            assert torch.equal(os_, torch.from_numpy(small).cuda())
