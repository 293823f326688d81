"""Build of the sm_100a shared library ``vox_b200/libvox_cuda.so`` (kernels + C ABI + C++ host wrappers).

Every ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` only and every ``csrc/*.cpp`` by the host compiler; the
objects are linked into one shared library with the CUDA runtime linked statically; at run time it needs the NVIDIA
driver and the toolkit's cuBLAS (the GEMMs of the F5 DiT step), found through an rpath to the toolkit's lib64.
Objects are rebuilt when their source or any header is newer.

Usage: ``python -m vox_b200.build [--force]``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libvox_cuda.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xptxas", "-warn-spills",
    f"-I{INCLUDE}",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the vox_cuda library needs the CUDA toolkit to build")


def cuda_include() -> str:
    return str(Path(nvcc()).resolve().parent.parent / "include")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + sorted(INCLUDE.glob("*.h")) + sorted(INCLUDE.glob("*.hpp"))


def _stale(src: Path, obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    if src.suffix == ".cu":
        cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [os.environ.get("CXX", "g++"), *CXX_FLAGS, f"-I{cuda_include()}", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link ``libvox_cuda.so`` for sm_100a; returns its path."""
    OBJ.mkdir(exist_ok=True)
    deps = _headers()
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    jobs = []
    for s in srcs:
        o = OBJ / (s.name + ".o")
        if force or _stale(s, o, deps):
            jobs.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for (s, _), err in zip(jobs, ex.map(lambda j: _compile(j[0], j[1], verbose), jobs)):
            if verbose and err.strip():
                print(f"[{s.name}]\n{err}", file=sys.stderr)
    objs = [OBJ / (s.name + ".o") for s in srcs]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cuda_lib = str(Path(nvcc()).resolve().parent.parent / "lib64")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs), f"-L{cuda_lib}", "-lcublas",
               "-Xlinker", f"-rpath,{cuda_lib}", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
