"""Writing Vox .tmod weight containers (the layout of src/formats.hpp:44-90, written as tmod_write does,
src/formats.cpp:215-249): a 64-byte header ("VOXM", version 1.0, flags, manifest and data ranges), the JSON manifest
with its "blobs" table {name: {dtype, shape, offset, nbytes}} (offsets relative to the data area, each blob aligned to
4096 bytes), zero padding to the 4096-aligned data area, then the blobs in name order. Reading and uploading are
vox_b200.Tmod (the C ABI's vox_cuda_tmod_*)."""

from __future__ import annotations

import json
import struct

import numpy as np

ALIGN = 4096
DTYPES = ["F32", "F16", "BF16", "I32", "I16", "I8", "U8"]  # Vox's DType order (src/common.hpp:22)
NUMPY = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I32": np.int32, "I16": np.int16, "I8": np.int8, "U8": np.uint8}


def _align(v: int) -> int:
    return (v + ALIGN - 1) // ALIGN * ALIGN


def write_tmod(path, manifest: dict, blobs: dict, flags: int = 0) -> None:
    """blobs: name -> (dtype name, shape, bytes). tmod_write (formats.cpp:215-249): blobs in sorted-name order."""
    table, off = {}, 0
    for name in sorted(blobs):
        dt, shape, data = blobs[name]
        off = _align(off)
        table[name] = {"dtype": dt, "shape": list(shape), "offset": off, "nbytes": len(data)}
        off += len(data)
    m = dict(manifest)
    m["blobs"] = table
    text = json.dumps(m, indent=2, sort_keys=True, ensure_ascii=False).encode()
    data_offset = _align(64 + len(text))
    hdr = struct.pack("<4sHHIIQQQQ16s", b"VOXM", 1, 0, flags, 0, 64, len(text), data_offset, off, bytes(16))
    with open(path, "wb") as f:
        f.write(hdr)
        f.write(text)
        f.write(bytes(data_offset - 64 - len(text)))
        pos = 0
        for name in sorted(blobs):
            data = blobs[name][2]
            a = _align(pos)
            f.write(bytes(a - pos))
            f.write(data)
            pos = a + len(data)
