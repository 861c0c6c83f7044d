"""Minimal safetensors reader/writer (no third-party dependency).

Mirrors what the reference's loader expects (src/main.zig:1259-1362,
2311-2404): an 8-byte little-endian header length, a JSON header mapping each
tensor name to ``{"dtype", "shape", "data_offsets"}``, then the raw data.
Reading memory-maps the file, like the reference, so a 614 MB checkpoint is
not copied before it is handed to the GPU library.
"""
from __future__ import annotations

import json
import struct
from typing import Dict, Tuple

import numpy as np

# dtype tag -> (numpy dtype used for the raw view, element size)
_DTYPES = {
    "F16": (np.uint16, 2),
    "BF16": (np.uint16, 2),
    "F32": (np.float32, 4),
}


class SafetensorsError(ValueError):
    """The file is not a safetensors image this library can read
    (the reference's error.BadSafetensors, src/main.zig:1359)."""


def read(path: str) -> Dict[str, Tuple[str, np.ndarray]]:
    """name -> (dtype tag, read-only numpy view of the mapped data)."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    if mm.size < 8:
        raise SafetensorsError("%s: shorter than the 8-byte header length" % path)
    (n,) = struct.unpack("<Q", bytes(mm[:8]))
    if n + 8 > mm.size:
        raise SafetensorsError("%s: header length %d exceeds file size" % (path, n))
    hdr = json.loads(bytes(mm[8:8 + n]))
    base = 8 + n
    out: Dict[str, Tuple[str, np.ndarray]] = {}
    for name, e in hdr.items():
        if name == "__metadata__":
            continue
        dt = e["dtype"]
        lo, hi = e["data_offsets"]
        raw = mm[base + lo: base + hi]
        if dt not in _DTYPES:
            out[name] = (dt, raw)
            continue
        npdt, size = _DTYPES[dt]
        if (hi - lo) % size:
            raise SafetensorsError("tensor %s has a byte length that is not a multiple of %d" % (name, size))
        out[name] = (dt, raw.view(npdt).reshape(e["shape"]))
    return out


def write(path: str, tensors: Dict[str, Tuple[str, np.ndarray]]) -> None:
    """Write ``name -> (dtype tag, array)``; arrays hold raw 16-bit patterns
    for F16/BF16 and float32 for F32."""
    hdr = {}
    off = 0
    order = list(tensors.keys())
    for name in order:
        dt, arr = tensors[name]
        nbytes = arr.size * _DTYPES[dt][1]
        hdr[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    blob = json.dumps(hdr, separators=(",", ":")).encode()
    blob += b" " * ((8 - len(blob) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for name in order:
            dt, arr = tensors[name]
            f.write(np.ascontiguousarray(arr).tobytes())
