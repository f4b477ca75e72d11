"""Test helper: writes safetensors files (8-byte little-endian header length,
JSON header, payload) and sharded checkpoints with an index, for the
checkpoint-loader tests."""
import json
import os
import struct

import numpy as np


def bf16_bytes(a: np.ndarray) -> bytes:
    return np.ascontiguousarray(a, dtype=np.uint16).astype("<u2").tobytes()


def write_safetensors(path, tensors, metadata=None, raw_header=None):
    """tensors: {name: (dtype, shape, payload bytes)}, laid out in order."""
    header, payload, off = {}, b"", 0
    for name, (dtype, shape, data) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        payload += data
        off += len(data)
    if metadata is not None:
        header["__metadata__"] = metadata
    hb = json.dumps(header).encode() if raw_header is None else raw_header
    hb += b" " * ((8 - len(hb) % 8) % 8)  # keep the payload 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        f.write(payload)


def write_checkpoint(directory, shards):
    """shards: {file name: {tensor name: bf16 array with its shape}}; writes
    the shards and model.safetensors.index.json."""
    os.makedirs(directory, exist_ok=True)
    weight_map = {}
    for fname, tensors in shards.items():
        write_safetensors(os.path.join(directory, fname),
                          {n: ("BF16", a.shape, bf16_bytes(a)) for n, a in tensors.items()})
        weight_map.update({n: fname for n in tensors})
    with open(os.path.join(directory, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": weight_map}, f)
