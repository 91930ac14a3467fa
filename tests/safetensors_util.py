"""Writes small synthetic .safetensors files for the convert tests."""
import json
import struct

import numpy as np

DT = {np.float32: "F32", np.float16: "F16", np.int32: "I32"}


def write_safetensors(path, tensors, metadata=None):
    """tensors: list of (name, dtype string, numpy array) in file order."""
    header, off, blobs = {}, 0, []
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dt, arr in tensors:
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    js = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(js)))
        f.write(js)
        for b in blobs:
            f.write(b)


def blob_bytes(f16_bits: np.ndarray) -> bytes:
    """The ANE blob the reference writes for fp16 data (core/safetensors.cpp:316-343)."""
    h = bytearray(128)
    h[0], h[4] = 1, 2
    h[64:68] = b"\xEF\xBE\xAD\xDE"
    h[68] = 1
    h[72:76] = struct.pack("<I", (f16_bits.size * 2) & 0xFFFFFFFF)
    h[80:84] = struct.pack("<I", 128)
    return bytes(h) + np.ascontiguousarray(f16_bits, np.uint16).tobytes()
