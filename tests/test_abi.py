"""CPU tests of the C ABI boundary: the shared library loads, exports every function include/vox_cuda.h declares,
and rejects bad arguments with VOX_CUDA_ERR_ARG and a message before touching the device (no kernel runs here)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "vox_cuda.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"VOX_CUDA_API\s+[\w\s\*]+?\b(vox_cuda_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from vox_b200 import build

    build.build()
    return ctypes.CDLL(str(build.LIB))


def test_header_declares_the_operator_set():
    names = declared_functions()
    for op in ("rmsnorm", "layernorm", "adaln", "gated_add", "bias_add", "softmax_rows", "silu_mul", "swiglu_fused", "gelu",
               "add", "mul", "snake", "dequant_q8", "dequant_q4", "row_reduce", "global_sum_partials", "global_sum_finish"):
        assert f"vox_cuda_{op}" in names


def test_library_exports_every_declared_symbol(lib):
    from vox_b200 import build

    out = subprocess.run(["nm", "-D", "--defined-only", str(build.LIB)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (vox_cuda_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"not exported: {missing}"
    for n in declared_functions():
        assert hasattr(lib, n)


def test_library_targets_sm100a_only():
    from vox_b200 import build

    out = subprocess.run(["cuobjdump", "--list-elf", str(build.LIB)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    archs = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert archs == {"100a"}, archs


def test_argument_errors_are_reported_without_a_device(lib):
    import vox_b200 as v

    with pytest.raises(v.VoxCudaError):
        v._check(v.lib.vox_cuda_rmsnorm(None, None, None, 4, 16, 1e-6, 7, None))  # bad dtype
    assert b"dtype" in v.lib.vox_cuda_last_error()
    assert v.lib.vox_cuda_rmsnorm(None, None, None, 4, 0, 1e-6, 0, None) == -6  # n = 0
    assert v.lib.vox_cuda_dequant_q8(None, None, 0, None, 1, 4, 33, None) == -6  # cols % 32 != 0
    assert b"multiple of 32" in v.lib.vox_cuda_last_error()
    assert v.lib.vox_cuda_snake(None, None, None, None, 16, 4, 1, 9, None) == -6  # unknown kind
    assert v.lib.vox_cuda_softmax_rows(None, None, 2, 8, 1.0, -1, 0, None) == -6
    assert v.lib.vox_cuda_adaln(None, None, None, None, None, None, 1, 1, 8, 1e-6, 1, None) == -6  # NULL x
    # gate and residual must come together
    assert v.lib.vox_cuda_adaln(1, 1, 1, 1, None, 1, 1, 1, 8, 1e-6, 1, None) == -6
    # a shard that does not start on a global-sum slot boundary
    assert v.lib.vox_cuda_global_sum_partials(1, 10, 4, 1, 8400, 1, 1, 0, None) == -6
    assert b"slots" in v.lib.vox_cuda_last_error()
    # empty work is a no-op, not an error
    assert v.lib.vox_cuda_add(None, None, None, 0, 0, None) == 0
    assert v.lib.vox_cuda_rmsnorm(None, None, None, 0, 16, 1e-6, 0, None) == 0


def test_last_error_is_per_thread(lib):
    import threading

    import vox_b200 as v

    v.lib.vox_cuda_gelu(None, None, 4, 9, 0, None)
    seen = {}

    def other():
        seen["msg"] = v.lib.vox_cuda_last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == b""
    assert b"kind" in v.lib.vox_cuda_last_error()


def test_version(lib):
    import vox_b200 as v

    assert v.version().startswith("vox-cuda") and "sm_100a" in v.version()


def test_fastdiv_host_arithmetic(tmp_path):
    """FastDiv (csrc/common.cuh), the invariant-divisor division every indexed kernel uses, against exact division."""
    src = tmp_path / "fd.cu"
    src.write_text(r'''
#include "common.cuh"
#include <cstdio>
#include <cstdint>
int main() {
    const uint32_t ds[] = {1u, 2u, 3u, 5u, 7u, 8u, 24u, 100u, 128u, 250u, 255u, 256u, 640u, 1000u, 3000u, 6000u, 24000u,
                           65535u, 65536u, 1000003u, 0x7fffffffu, 0x80000000u, 0xfffffffeu, 0xffffffffu};
    uint64_t bad = 0, x = 88172645463325252ull;
    for (uint32_t d : ds) {
        voxcuda::FastDiv f(d);
        const uint32_t ns[] = {0u, 1u, d - 1u, d, d + 1u, 2u * d, 0xffffffffu, 0xfffffffeu, 0x80000000u};
        for (uint32_t n : ns) if (f.div(n) != n / d || f.mod(n) != n % d) ++bad;
        for (int i = 0; i < 200000; ++i) {
            x ^= x << 13; x ^= x >> 7; x ^= x << 17;
            const uint32_t n = uint32_t(x);
            if (f.div(n) != n / d) ++bad;
        }
    }
    std::printf("%llu\n", (unsigned long long)bad);
    return bad != 0;
}
''')
    from vox_b200 import build

    exe = tmp_path / "fd"
    subprocess.run([build.nvcc(), *build.ARCH, "-std=c++17", f"-I{build.CSRC}", f"-I{build.INCLUDE}", str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "0", r.stdout
