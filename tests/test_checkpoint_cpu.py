"""Safetensors validation of the checkpoint loader (fw_checkpoint.cu), on
CPU through the handle-free fw_safetensors_tensor_info: the checks the
reference's mapped-shard reader makes (src/checkpoint_catalog.rs:146-253)
each reject a malformed file with FW_EINVAL, and a well-formed one reports
dtype, shape and payload range."""
import json
import struct

import numpy as np
import pytest

import firewing_b200 as fw
from st_writer import bf16_bytes, write_safetensors


def info(path, name):
    return fw.safetensors_tensor_info(str(path), name)


def test_reports_dtype_shape_and_range(tmp_path):
    a = np.arange(6, dtype=np.uint16).reshape(2, 3)
    b = np.zeros(4, dtype=np.float32)
    p = tmp_path / "m.safetensors"
    write_safetensors(p, {"w": ("BF16", [2, 3], bf16_bytes(a)), "v": ("F32", [4], b.tobytes())},
                      metadata={"format": "pt"})
    assert info(p, "w") == {"dtype": "BF16", "shape": [2, 3], "offset": 0, "bytes": 12}
    assert info(p, "v") == {"dtype": "F32", "shape": [4], "offset": 12, "bytes": 16}


def _expect_invalid(p, name="w", match=None):
    with pytest.raises(fw.FwError) as e:
        info(p, name)
    assert e.value.code == fw.FW_EINVAL
    if match:
        assert match in str(e.value), str(e.value)


def _raw(p, header: bytes, payload: bytes = b"", length=None):
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(header) if length is None else length))
        f.write(header)
        f.write(payload)


def test_rejects_malformed_files(tmp_path):
    p = tmp_path / "bad.safetensors"
    good = {"w": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}}
    hdr = json.dumps(good).encode()
    _raw(p, b"{}", length=0)
    _expect_invalid(p, match="too short")
    _raw(p, hdr + b" " * 8, b"\0" * 4, length=0)
    _expect_invalid(p, match="invalid safetensors header")
    _raw(p, hdr, b"\0" * 4, length=len(hdr) + 100)
    _expect_invalid(p, match="invalid safetensors header")
    _raw(p, b"[1, 2, 3]     ", b"\0" * 4)
    _expect_invalid(p, match="not an object")
    _raw(p, b'{"w": {"dtype": "BF16", ', b"\0" * 8)
    _expect_invalid(p, match="header")
    for entry, msg in [({"dtype": "Q7", "shape": [2], "data_offsets": [0, 4]}, "unknown dtype"),
                       ({"dtype": "BF16", "shape": [2, 0], "data_offsets": [0, 0]}, "empty shape"),
                       ({"dtype": "BF16", "shape": [], "data_offsets": [0, 2]}, "empty shape"),
                       ({"dtype": "BF16", "shape": [3], "data_offsets": [0, 4]}, "payload layout"),
                       ({"dtype": "BF16", "shape": [4], "data_offsets": [0, 8]}, "payload layout"),
                       ({"dtype": "BF16", "shape": [2], "data_offsets": [0]}, "invalid offsets"),
                       ({"dtype": "BF16", "shape": [-2], "data_offsets": [0, 4]}, "invalid shape"),
                       ({"shape": [2], "data_offsets": [0, 4]}, "missing dtype")]:
        _raw(p, json.dumps({"w": entry}).encode(), b"\0" * 4)
        _expect_invalid(p, match=msg)
    two = {"w": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]},
           "v": {"dtype": "BF16", "shape": [2], "data_offsets": [2, 6]}}
    _raw(p, json.dumps(two).encode(), b"\0" * 8)
    _expect_invalid(p, match="overlapping")
    dup = b'{"w": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}, ' \
          b'"w": {"dtype": "BF16", "shape": [2], "data_offsets": [4, 8]}}'
    _raw(p, dup, b"\0" * 8)
    _expect_invalid(p, match="duplicate")
    meta = {"__metadata__": [1], **good}
    _raw(p, json.dumps(meta).encode(), b"\0" * 4)
    _expect_invalid(p, match="__metadata__")
    _raw(p, hdr, b"\0" * 4)
    _expect_invalid(p, name="absent", match="absent")
    _expect_invalid(tmp_path / "missing.safetensors", match="cannot open")


def test_json_escapes_and_numbers(tmp_path):
    p = tmp_path / "esc.safetensors"
    name = 'a"b\\c/é\U0001f600'
    write_safetensors(p, {name: ("BF16", [1], b"\0\0")})
    assert info(p, name)["bytes"] == 2
    # offsets must be exact non-negative integers
    _raw(p, b'{"w": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2.0]}}', b"\0\0")
    _expect_invalid(p, match="invalid end")
