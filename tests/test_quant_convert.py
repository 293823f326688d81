"""CPU checks of the arithmetic behind the f16 weight conversions of the quantized prefill GEMM (vox_b200/csrc/gemm.cu:
the converter warps of gemm_q_kernel and q_w_to_f16_kernel), emulated with numpy's IEEE half type.

Both write W as f16(code) * f16(scale) with one rounding: a code byte placed under the exponent pattern 0x64 is the
half 1024 + u exactly, subtracting 1024 + offset (128 for Q8 codes stored as code ^ 0x80, 8 for Q4 nibbles) leaves the
integer code exactly, and the product of an integer of at most 8 bits with a half scale is exact in f32 before its
rounding to half. The tests check those identities over every code, the Q4 nibble order the weight pass reads (Vox's
layout, kernels.cpp:453-463: byte j of a 16-byte block holds element j in its low nibble and element j + 16 in its high
nibble) against the oracle's dequantisation, and the distance of the f16 weights from Vox's f32 ones (the error
budget of the GEMM tests).
"""

from __future__ import annotations

import numpy as np


def _half_bits(b):
    return np.asarray(b, dtype=np.uint16).view(np.float16)


def test_exponent_pattern_gives_every_code_exactly():
    u = np.arange(256, dtype=np.uint16)
    assert np.array_equal(_half_bits(0x6400 | u).astype(np.float32), 1024.0 + u)
    q8 = np.arange(-128, 128)
    b8 = (q8 & 0xFF) ^ 0x80  # the stored byte with its sign bit flipped: code + 128
    got8 = _half_bits(0x6400 | b8) - np.float16(1152)  # f16x2 (1152, 1152): 1024 + 128
    assert got8.dtype == np.float16 and np.array_equal(got8.astype(np.float32), q8)
    n4 = np.arange(16)
    got4 = _half_bits(0x6400 | n4) - np.float16(1032)  # 1024 + 8: Q4 codes are the nibble minus 8
    assert np.array_equal(got4.astype(np.float32), n4 - 8)


def test_code_times_half_scale_rounds_once(port):
    rng = np.random.default_rng(3)
    scales = np.concatenate([port.uniform_arr((4096,), 0.001, 0.05, sid=300), rng.uniform(1e-6, 511.0, 1024).astype(np.float32),
                             np.array([2.0 ** -14, 2.0 ** -24, 5.96e-8, 511.0, 1.0], np.float32)])  # |code * scale| < 65504
    s16 = scales.astype(np.float16)  # __float2half_rn of an f32 scale (f16 scales pass unchanged)
    codes = np.arange(-128, 128, dtype=np.float32)
    c16 = codes.astype(np.float16)
    # mul.rn.f16x2: the exact product (at most 8 x 11 significant bits, exact in f32) rounded once to half
    kernel = (c16[:, None].astype(np.float32) * s16[None, :].astype(np.float32)).astype(np.float16)
    exact = (codes[:, None].astype(np.float64) * s16[None, :].astype(np.float64)).astype(np.float16)
    assert np.array_equal(kernel.view(np.uint16), exact.view(np.uint16))


def _weight_pass_q4_codes(q):
    """q_w_to_f16_kernel's reading of Q4 bytes [rows][cols / 2]: eight weights e .. e + 7 a thread (e a multiple of 8
    in the flat [rows][cols] order), from the bytes blk * 16 + (e % 16) .. + 7 of their 32-block blk = e / 32, low
    nibbles where e % 32 < 16, high nibbles above."""
    flat = q.reshape(-1)
    n = flat.size * 2
    out = np.empty(n, np.int32)
    for e in range(0, n, 8):
        blk, p = e >> 5, e & 31
        v = flat[blk * 16 + (p & 15): blk * 16 + (p & 15) + 8].astype(np.int32)
        out[e:e + 8] = ((v >> (0 if p < 16 else 4)) & 0xF) - 8
    return out.reshape(q.shape[0], q.shape[1] * 2)


def test_weight_pass_reads_q4_in_vox_order(port):
    rows, cols = 6, 256
    q = port.fill_u8((rows, cols // 2), sid=310)
    ones = np.ones((rows, cols // 32), np.float32)
    assert np.array_equal(_weight_pass_q4_codes(q).astype(np.float32), port.dequant_q4(q, ones))


def test_f16_weights_stay_within_the_gemm_error_budget(port):
    """code * scale rounded to half (after the scale's own rounding) is within 2^-10 of Vox's f32 weight, relative,
    for normal results: the per-product share of the 1.5e-3 * sum |w x| bound of the GEMM tests."""
    rows, cols = 64, 512
    q8 = port.fill_i8((rows, cols), -128, 127, sid=320)
    sc = port.uniform_arr((rows, cols // 32), 0.001, 0.05, sid=321)
    vox_w = port.dequant_q8(q8, sc).astype(np.float64)
    s16 = np.repeat(sc.astype(np.float16).astype(np.float32), 32, axis=1)
    w16 = (q8.astype(np.float32) * s16).astype(np.float16).astype(np.float64)
    assert np.all(np.abs(w16 - vox_w) <= 2.0 ** -10 * np.abs(vox_w) + 1e-30)
