"""The C++17 host seam (include/vox_gpu_cuda.hpp): build the C++ test program against libvox_cuda.so and the oracle,
and run it on the GPU (tests/cpp/test_gpu_cuda.cpp)."""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def build_cpp_test(tmp: Path) -> Path:
    from oracle.oracle import build_port
    from vox_b200 import build

    build.build()
    port = build_port()
    exe = tmp / "test_gpu_cuda"
    cmd = [os.environ.get("CXX", "g++"), "-std=c++17", "-O2", "-Wall", f"-I{ROOT / 'include'}", str(ROOT / "tests/cpp/test_gpu_cuda.cpp"),
           str(build.LIB), str(port), f"-Wl,-rpath,{build.LIB.parent}:{port.parent}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_cpp_seam_compiles_and_links(tmp_path):
    assert build_cpp_test(tmp_path).exists()


@pytest.mark.gpu
def test_cpp_seam_on_gpu(tmp_path, vox):
    exe = build_cpp_test(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "OK" in r.stdout
