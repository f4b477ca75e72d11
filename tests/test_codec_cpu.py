"""Compressed expert containers on CPU (fw_codec_container_check): the
manifest and frame checks, zstd decoding and both SHA-256 digests of the
reference's container format, against containers written with libzstd and
hashlib."""
import json

import numpy as np
import pytest

import firewing_b200 as fw
from codec_writer import expert_source, write_container

SRC = 3 * 256 * 128 * 2  # the test block's expert: gate_up [256][256] + down [256][128]


def experts(n, seed=0):
    rng = np.random.default_rng(seed)
    out = {}
    for i in range(n):
        gu = rng.integers(0, 1 << 16, size=(256, 256), dtype=np.uint16)
        gu &= 0xBFFF  # plausible bf16 magnitudes (compressible high bytes)
        dn = rng.integers(0, 1 << 16, size=(256, 128), dtype=np.uint16) & 0xBFFF
        out[(i % 2, 3 * i)] = expert_source(gu, dn)
    return out


def test_decodes_and_verifies(tmp_path):
    m = write_container(tmp_path, experts(5))
    assert fw.codec_container_check(m, -1, SRC) == 5
    assert fw.codec_container_check(m, 0, SRC) == 3
    assert fw.codec_container_check(m, 1, SRC, verify=False) == 2


def _edit(m, fn):
    with open(m) as f:
        d = json.load(f)
    fn(d)
    with open(m, "w") as f:
        json.dump(d, f)


@pytest.mark.parametrize("edit,msg", [
    (lambda d: d.update(exact_transform="bf16_identity"), "exact_transform"),
    (lambda d: d["codec"].update(name="lz4"), "codec"),
    (lambda d: d.update(container_file="../x"), "container_file"),
    (lambda d: d["records"][1].update(offset=d["records"][1]["offset"] + 8), "page-aligned"),
    (lambda d: d["records"][0].update(physical_bytes=1 << 40), "outside"),
    (lambda d: d["records"][0].update(source_sha256="0" * 64), "source hash"),
    (lambda d: d["records"][0].update(frame_sha256="f" * 64), "frame hash"),
    (lambda d: d["records"][0].update(frame_sha256="xyz"), "invalid record"),
])
def test_rejects_bad_manifests(tmp_path, edit, msg):
    m = write_container(tmp_path, experts(3))
    _edit(m, edit)
    with pytest.raises(fw.FwError) as e:
        fw.codec_container_check(m, -1, SRC)
    assert e.value.code == fw.FW_EINVAL and msg in str(e.value), str(e.value)


def test_rejects_wrong_expert_size_and_corrupt_frames(tmp_path):
    m = write_container(tmp_path, experts(2))
    with pytest.raises(fw.FwError) as e:
        fw.codec_container_check(m, -1, SRC + 2)
    assert "source_bytes_per_expert" in str(e.value)
    # corrupt one byte of the first frame: the frame hash catches it; without
    # verification zstd's own checks or the size check still reject it
    blob = bytearray((tmp_path / "experts.container").read_bytes())
    blob[40] ^= 0xFF
    (tmp_path / "experts.container").write_bytes(bytes(blob))
    with pytest.raises(fw.FwError) as e:
        fw.codec_container_check(m, -1, SRC)
    assert "frame hash" in str(e.value)
