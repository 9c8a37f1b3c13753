"""Writes safetensors shards for the checkpoint tests: u64 little-endian header
length, JSON header {name: {dtype, shape, data_offsets}} (+ __metadata__),
then the tensors' bytes back to back."""
import json
import struct

import numpy as np


def encode(tensors: dict, metadata: dict | None = None) -> bytes:
    """tensors: name -> (dtype name, shape, little-endian bytes)."""
    header, blobs, off = {}, [], 0
    for name, (dt, shape, raw) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata is not None:
        header["__metadata__"] = metadata
    text = json.dumps(header).encode()
    text += b" " * (-len(text) % 8)
    return struct.pack("<Q", len(text)) + text + b"".join(blobs)


def write(path, tensors: dict, metadata: dict | None = None) -> None:
    with open(path, "wb") as f:
        f.write(encode(tensors, metadata))


def bf16(bits: np.ndarray, shape) -> tuple:
    return ("BF16", tuple(shape), np.ascontiguousarray(bits, "<u2").tobytes())


def f16(x: np.ndarray, shape) -> tuple:
    return ("F16", tuple(shape), np.ascontiguousarray(x, "<f2").tobytes())


def f32(x: np.ndarray, shape) -> tuple:
    return ("F32", tuple(shape), np.ascontiguousarray(x, "<f4").tobytes())
