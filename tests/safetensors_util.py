"""Writes .safetensors files for the tests (the published layout: u64
little-endian header length, JSON header of dtype / shape / data_offsets per
tensor, then the raw little-endian data), and the bf16 rounding the engine
applies on load."""

import json
import struct

import numpy as np


def bf16_bits(a):
    """fp32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(np.asarray(a, np.float32)).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def encode(a, dtype):
    """(safetensors dtype name, raw bytes) of fp32 array a stored as dtype ("BF16", "F16", "F32")."""
    if dtype == "BF16":
        return dtype, bf16_bits(a).tobytes()
    if dtype == "F16":
        return dtype, np.asarray(a, np.float32).astype(np.float16).tobytes()
    return "F32", np.ascontiguousarray(np.asarray(a, np.float32)).tobytes()


def as_loaded(a, dtype):
    """The bf16 bits the engine holds after loading fp32 array a stored as dtype."""
    if dtype == "F16":
        a = np.asarray(a, np.float32).astype(np.float16).astype(np.float32)
    return bf16_bits(a)


def write(path, tensors, dtype):
    """tensors: iterable of (name, fp32 array); every tensor stored as dtype."""
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, a in tensors:
        dt, raw = encode(a, dtype)
        header[name] = {"dtype": dt, "shape": list(np.shape(a)), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)  # keep the data section 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
