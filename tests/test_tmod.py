"""The .tmod reader of the C ABI (vox_cuda_tmod_open / _count / _name / _info / _data) on CPU: the golden file written
by the reference's own tmod_write (formats.cpp:215-249) reads back blob for blob; the format checks of
TmodFile::TmodFile (formats.cpp:175-205) reject broken files with VOX_ERR_FORMAT / VOX_ERR_IO; files from the test
writer (oracle/tmod.py) read the same in this reader and in the reference's."""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLD = ROOT / "tests" / "golden" / "tiny.tmod"


def test_golden_tmod_reads_back(vox_lib, golden):
    vox = vox_lib
    g = golden["tmod"]
    with vox.Tmod(GOLD) as t:
        assert sorted(t.names()) == ["emb", "layer.u", "layer.u.scale", "layer.w", "layer.w.scale", "norm"]
        assert t.info("layer.w") == ("I8", (48, 64), 48 * 64)
        assert t.info("layer.u") == ("U8", (16, 32), 16 * 32)
        assert t.info("emb") == ("BF16", (3, 8), 48)
        assert t.host_bytes("layer.w") == g["q8"].tobytes()
        assert t.host_bytes("layer.u") == g["q4"].tobytes()
        assert t.host_bytes("layer.w.scale") == g["s8"].tobytes()
        assert t.host_bytes("layer.u.scale") == g["s4"].tobytes()
        assert t.host_bytes("norm") == g["norm"].tobytes()
        assert t.host_bytes("emb") == g["emb"].tobytes()
        with pytest.raises(vox.VoxCudaError) as e:
            t.info("missing")
        assert e.value.status == -2


def _broken(tmp_path, name, mutate):
    raw = bytearray(GOLD.read_bytes())
    mutate(raw)
    p = tmp_path / name
    p.write_bytes(bytes(raw))
    return p


@pytest.mark.parametrize("case", ["magic", "version", "manifest_range", "json", "blob_range", "truncated"])
def test_broken_files_are_rejected(vox_lib, tmp_path, case):
    vox = vox_lib
    def mutate(raw):
        mo, ms, do, ds = struct.unpack_from("<QQQQ", raw, 16)
        if case == "magic":
            raw[0:4] = b"VOXX"
        elif case == "version":
            struct.pack_into("<H", raw, 4, 2)
        elif case == "manifest_range":
            struct.pack_into("<Q", raw, 24, len(raw))
        elif case == "json":
            raw[mo + ms - 1:mo + ms] = b","  # the closing brace of the manifest
        elif case == "blob_range":
            struct.pack_into("<Q", raw, 40, 100)  # data_size: smaller than the blobs
        elif case == "truncated":
            del raw[len(raw) - 4096:]
    p = _broken(tmp_path, f"{case}.tmod", mutate)
    with pytest.raises(vox.VoxCudaError) as e:
        vox.Tmod(p)
    assert e.value.status == -2, e.value


def test_missing_file_is_io_error(vox_lib, tmp_path):
    vox = vox_lib
    with pytest.raises(vox.VoxCudaError) as e:
        vox.Tmod(tmp_path / "none.tmod")
    assert e.value.status == -1


def test_test_writer_matches_reference_reader(vox_lib, tmp_path):
    vox = vox_lib
    from oracle.oracle import ref
    from vox_b200.tmodfile import write_tmod

    rng = np.random.default_rng(3)
    blobs = {"w": ("I8", (33, 64), rng.integers(-128, 128, (33, 64), dtype=np.int8).tobytes()),
             "w.scale": ("F32", (33, 2), rng.random((33, 2), dtype=np.float32).tobytes()),
             "empty": ("F32", (0,), b""), "v": ("F16", (5,), rng.random(5).astype(np.float16).tobytes())}
    p = tmp_path / "t.tmod"
    write_tmod(p, {"family": "t", "nested": {"a": [1, {"b": "é\\n"}]}}, blobs)
    with vox.Tmod(p) as t:
        for n, (dt, shape, data) in blobs.items():
            assert t.info(n) == (dt, shape, len(data))
            assert t.host_bytes(n) == data
    from oracle.tmod import read_tmod

    _, back = read_tmod(p)
    assert {n: (dt, tuple(sh), d) for n, (dt, sh, d) in back.items()} == {n: (dt, tuple(sh), d) for n, (dt, sh, d) in blobs.items()}
    R = ref()
    if R is not None:
        for n, (_, _, data) in blobs.items():
            assert R.tmod_read(p, n) == data
