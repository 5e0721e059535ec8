"""Writes .safetensors files for the loader tests (the format: u64
little-endian header length, JSON header, raw little-endian tensor bytes)."""
import json
import struct

import numpy as np

import synthetic as S


def write_safetensors(path, tensors, metadata=None):
    """tensors: {name: (array, dtype)} with dtype "F32", "BF16" (array holds
    bf16-exact float32 values), "F16" or "I64"."""
    header, blobs, off = {}, [], 0
    for name, (a, dt) in tensors.items():
        a = np.asarray(a)
        if dt == "F32":
            raw = np.ascontiguousarray(a, np.float32).tobytes()
        elif dt == "BF16":
            raw = np.ascontiguousarray(S.bf16_bits(np.asarray(a, np.float32)), np.uint16).tobytes()
        elif dt == "F16":
            raw = np.ascontiguousarray(a, np.float16).tobytes()
        elif dt == "I64":
            raw = np.ascontiguousarray(a, np.int64).tobytes()
        else:
            raise ValueError(dt)
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
