"""The tcgen05 GEMM (vox_cuda_gemm_bf16) through the C ABI against a plain PyTorch fp32 reference of the same op.

y = act(x . w^T + bias) with bf16 x and w: every product of two bf16 values is exact in f32, so the GEMM differs
from the fp32 reference on the same (bf16-valued) operands only by the order of its f32 sums: within 1e-5 of
sum |x w| per element (f32 output); a bf16 output adds one rounding (2^-8 relative). Shapes cover one row, edges
that are not multiples of the 128 x BN tiles, K that is not a multiple of the 64-element step (zero fill), the
F5-base projections, and every tile kernel forced in turn (one CTA: 64 / 128 / 256 columns; CTA pairs: 256 x 128,
256 x 192 and 256 x 256) on ragged shapes with each epilogue.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w, bias, act):
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias
    if act == 1:
        y = torch.nn.functional.gelu(y)
    elif act == 2:
        y = torch.nn.functional.gelu(y, approximate="tanh")
    return y


def _bound(x, w, bias):
    b = x.float().abs() @ w.float().abs().t()
    if bias is not None:
        b = b + bias.abs()
    return b


@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (100, 100, 712), (257, 257, 136), (300, 1000, 2048), (2048, 3072, 1024),
                                   (512, 12288, 4096), (2048, 1024, 2048), (130, 520, 64), (1000, 1000, 520), (777, 4100, 1024)])
def test_gemm_bf16_matches_fp32_reference(vox, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    want = _ref(x, w, bias, 0)
    bound = _bound(x, w, bias)
    got = vox.gemm_bf16(x, w, bias)
    torch.cuda.synchronize()
    assert ((got - want).abs() <= 1e-5 * bound + 1e-6).all(), f"max err {(got - want).abs().max().item()}"
    got_b = vox.gemm_bf16(x, w, bias, out_dtype=torch.bfloat16).float()
    assert ((got_b - want).abs() <= 4e-3 * want.abs() + 1e-5 * bound + 1e-6).all()
    # no bias, twice in a row (deterministic)
    a1, a2 = vox.gemm_bf16(x, w), vox.gemm_bf16(x, w)
    assert torch.equal(a1, a2)
    assert ((a1 - _ref(x, w, None, 0)).abs() <= 1e-5 * _bound(x, w, None) + 1e-6).all()
    assert vox.device_error() == 0


@pytest.mark.parametrize("act", [1, 2])
def test_gemm_bf16_gelu_epilogues(vox, act):
    m, n, k = 333, 640, 512
    g = torch.Generator(device="cuda").manual_seed(act)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    want = _ref(x, w, bias, act)
    bound = _bound(x, w, bias)
    got = vox.gemm_bf16(x, w, bias, act=act)
    torch.cuda.synchronize()
    # GELU's own approximation (A&S 26.2.17 / SFU tanh): within 1e-6 absolute of the exact function
    assert ((got - want).abs() <= 1e-5 * bound + 2e-6).all(), f"max err {(got - want).abs().max().item()}"
    got_b = vox.gemm_bf16(x, w, bias, act=act, out_dtype=torch.bfloat16).float()
    assert ((got_b - want).abs() <= 4e-3 * want.abs() + 1e-5 * bound + 2e-6).all()


def test_gemm_bf16_rejects_bad_operands(vox):
    x = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")  # k % 8 != 0
    w = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(vox.VoxCudaError):
        vox.gemm_bf16(x, w)
    with pytest.raises(vox.VoxCudaError):
        vox.gemm_bf16(x.float(), w)
    assert vox.device_error() == 0


@pytest.mark.parametrize("pair,bn", [(0, 64), (0, 128), (0, 256), (1, 128), (1, 192), (1, 256)])
@pytest.mark.parametrize("m,n,k", [(1000, 1000, 520), (300, 776, 136), (2048, 3072, 1024)])
def test_gemm_bf16_every_tile_kernel(vox, monkeypatch, pair, bn, m, n, k):
    """The tile selection is an estimate; each kernel it can pick is checked here on its own (the overrides are read
    at every call)."""
    monkeypatch.setenv("VOX_CUDA_GEMM_PAIR", str(pair))
    monkeypatch.setenv("VOX_CUDA_GEMM_BN", str(bn))
    g = torch.Generator(device="cuda").manual_seed(m + n + k + bn)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    bound = _bound(x, w, bias)
    for act in (0, 2):
        want = _ref(x, w, bias, act)
        got = vox.gemm_bf16(x, w, bias, act=act)
        torch.cuda.synchronize()
        assert ((got - want).abs() <= 1e-5 * bound + 2e-6).all(), f"act {act}: max err {(got - want).abs().max().item()}"
        got_b = vox.gemm_bf16(x, w, bias, act=act, out_dtype=torch.bfloat16).float()
        assert ((got_b - want).abs() <= 4e-3 * want.abs() + 1e-5 * bound + 2e-6).all()
    assert vox.device_error() == 0
