"""Test helper: writes compressed expert containers in the reference's
format (tools/build_sequential_shuffle_container.py): per expert, the
gate_up then down bytes, BF16-shuffled (even bytes, then odd bytes), one
independent zstd level-1 frame (libzstd through ctypes) at a page-aligned
offset, and a JSON manifest of the records with SHA-256 digests (hashlib)."""
import ctypes
import hashlib
import json
import os

import numpy as np

PAGE = 16384


def _zstd():
    z = ctypes.CDLL("libzstd.so.1")
    z.ZSTD_compressBound.restype = ctypes.c_size_t
    z.ZSTD_compressBound.argtypes = [ctypes.c_size_t]
    z.ZSTD_compress.restype = ctypes.c_size_t
    z.ZSTD_compress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    z.ZSTD_isError.restype = ctypes.c_uint
    z.ZSTD_isError.argtypes = [ctypes.c_size_t]
    return z


def compress(data: bytes, level: int = 1) -> bytes:
    z = _zstd()
    cap = z.ZSTD_compressBound(len(data))
    out = ctypes.create_string_buffer(cap)
    n = z.ZSTD_compress(out, cap, data, len(data), level)
    assert not z.ZSTD_isError(n)
    return out.raw[:n]


def shuffle_bf16(source: bytes) -> bytes:
    return source[0::2] + source[1::2]


def expert_source(gate_up: np.ndarray, down: np.ndarray) -> bytes:
    return np.ascontiguousarray(gate_up, dtype="<u2").tobytes() + np.ascontiguousarray(down, dtype="<u2").tobytes()


def write_container(directory, experts, page=PAGE, name="experts.container"):
    """experts: {(layer, expert): source bytes}.  Returns the manifest path."""
    os.makedirs(directory, exist_ok=True)
    records, blob = [], b""
    per = None
    for (layer, expert), source in sorted(experts.items()):
        per = len(source) if per is None else per
        frame = compress(shuffle_bf16(source))
        phys = (len(frame) + page - 1) // page * page
        records.append({"identity": f"{layer}:{expert}", "layer": layer, "expert": expert, "offset": len(blob),
                        "compressed_bytes": len(frame), "physical_bytes": phys,
                        "frame_sha256": hashlib.sha256(frame).hexdigest(),
                        "source_sha256": hashlib.sha256(source).hexdigest()})
        blob += frame + bytes(phys - len(frame))
    with open(os.path.join(directory, name), "wb") as f:
        f.write(blob)
    manifest = {"schema_version": 1, "codec": {"name": "zstandard", "level": 1, "independent_frames": True},
                "exact_transform": "bf16_even_bytes_then_odd_bytes_per_expert", "page_bytes": page,
                "source_bytes_per_expert": per, "records": records, "container_file": name}
    path = os.path.join(directory, "manifest.json")
    with open(path, "w") as f:
        json.dump(manifest, f)
    return path
