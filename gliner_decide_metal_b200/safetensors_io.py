"""Minimal safetensors reader / writer over numpy.

The reference keeps weights, inputs and logits in safetensors files
(``Weights.swift:26-28``, ``DeBERTa.swift:40-57``, ``main.swift:280-283,314-320``).
The C-ABI library parses weight files itself; this module is the Python side used to
write model files, to read and write ``DecisionInput`` files and to save logits.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

_DTYPES = {
    "F16": np.float16, "F32": np.float32, "F64": np.float64, "BF16": None,
    "I64": np.int64, "I32": np.int32, "I16": np.int16, "I8": np.int8,
    "U8": np.uint8, "BOOL": np.bool_,
}
_NAMES = {np.dtype(v): k for k, v in _DTYPES.items() if v is not None}


def save_file(tensors: dict, path, metadata: dict | None = None) -> None:
    """Write ``tensors`` (name -> numpy array) as one safetensors file; data is laid out
    in insertion order, 8-byte aligned header."""
    header = {}
    offset = 0
    arrays = []
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        if a.dtype not in _NAMES:
            raise TypeError(f"unsupported dtype {a.dtype} for {name}")
        nbytes = a.nbytes
        header[name] = {"dtype": _NAMES[a.dtype], "shape": list(a.shape),
                        "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
        arrays.append(a)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for a in arrays:
            f.write(a.tobytes(order="C"))


def load_file(path) -> dict:
    """Read every tensor of a safetensors file into numpy arrays (BF16 widened to F32)."""
    data = Path(path).read_bytes()
    (n,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + n])
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        b, e = info["data_offsets"]
        buf = data[base + b: base + e]
        if info["dtype"] == "BF16":
            u = np.frombuffer(buf, dtype=np.uint16).astype(np.uint32) << 16
            arr = u.view(np.float32)
        else:
            arr = np.frombuffer(buf, dtype=_DTYPES[info["dtype"]])
        out[name] = arr.reshape(info["shape"]).copy()
    return out
