"""safetensors reading and writing for the tests (TEST INFRASTRUCTURE ONLY).

read_tensor_f32 restates WeightStore::tensor_f32 (crates/voxtral/src/weights.rs:49-93)
with numpy: F32 bytes as little-endian f32, BF16 widened by bits << 16, any
other dtype refused.  write_safetensors lays a file out as the format
requires (8-byte little-endian header length, JSON header padded with spaces
to a multiple of 8, tensors back to back in the given order); the
reference's tests make their fixtures the same way with serialize_to_file
(weights.rs:106-193).
"""
from __future__ import annotations

import json
import struct

import numpy as np

SIZES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E5M2": 1, "F8_E4M3": 1, "I16": 2, "U16": 2, "F16": 2, "BF16": 2,
         "I32": 4, "U32": 4, "F32": 4, "F64": 8, "I64": 8, "U64": 8}


def write_safetensors(path, tensors, metadata=None):
    """tensors: list of (name, dtype, shape, raw bytes)."""
    header, offset, blobs = {}, 0, []
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [offset, offset + len(raw)]}
        offset += len(raw)
        blobs.append(raw)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_header(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    header.pop("__metadata__", None)
    return header, data


def read_tensor_f32(path, name):
    """weights.rs:49-93 -> (shape, f32 array)."""
    header, data = read_header(path)
    info = header[name]
    raw = data[info["data_offsets"][0]:info["data_offsets"][1]]
    if info["dtype"] == "F32":
        return info["shape"], np.frombuffer(raw, "<f4").astype(np.float32)
    if info["dtype"] == "BF16":
        bits = np.frombuffer(raw, "<u2").astype(np.uint32) << 16
        return info["shape"], bits.view(np.float32)
    raise ValueError(f"unsupported dtype for {name}: {info['dtype']}")
