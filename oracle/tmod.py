"""TEST INFRASTRUCTURE — a restatement of Vox's .tmod reader (TmodFile, src/formats.cpp:175-205) in Python, the
independent check of the product's reader (vox_cuda_tmod_open) and writer (vox_b200.tmodfile). Not product code."""

from __future__ import annotations

import json
import struct


def read_tmod(path) -> tuple[dict, dict]:
    """TmodFile (formats.cpp:175-205): returns (manifest, {name: (dtype, shape, bytes)})."""
    raw = open(path, "rb").read()
    magic, vmaj, _, _, _, mo, ms, do, ds, _ = struct.unpack("<4sHHIIQQQQ16s", raw[:64])
    assert magic == b"VOXM" and vmaj == 1
    manifest = json.loads(raw[mo:mo + ms].decode())
    out = {}
    for name, b in manifest.get("blobs", {}).items():
        out[name] = (b["dtype"], tuple(b["shape"]), raw[do + b["offset"]:do + b["offset"] + b["nbytes"]])
    return manifest, out
