"""add_bf16 (src/expert.rs:578) on the GPU (fw_add_bf16, the packed bf16
add the combine uses) against the f32 path bit for bit: the f32 sum of the
two widened values rounded to bf16 (round to nearest even, NaN as 0x7fc0),
over random bit patterns and the edge cases (signed zeros, subnormals,
infinities, NaNs, exponent gaps, rounding ties)."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402


def reference(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    fa = (a.astype(np.uint32) << 16).view(np.float32)
    fb = (b.astype(np.uint32) << 16).view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):  # infinities and NaNs on purpose
        u = (fa + fb).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r[nan] = 0x7FC0
    return r.astype(np.uint16)


def run(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    da = torch.from_numpy(a.view(np.int16)).cuda()
    db = torch.from_numpy(b.view(np.int16)).cuda()
    out = torch.empty_like(da)
    fw.add_bf16(da, db, a.size, out)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)


def test_random_bit_patterns():
    rng = np.random.default_rng(3)
    n = 1 << 22
    a = rng.integers(0, 1 << 16, n, dtype=np.uint32).astype(np.uint16)
    b = rng.integers(0, 1 << 16, n, dtype=np.uint32).astype(np.uint16)
    assert np.array_equal(run(a, b), reference(a, b))


def test_edge_cases_and_the_cpu_oracle():
    special = np.array([0x0000, 0x8000, 0x0001, 0x8001, 0x007F, 0x0080, 0x807F, 0x7F7F, 0xFF7F, 0x7F80, 0xFF80,
                        0x7FC0, 0x7F81, 0xFFC1, 0x3F80, 0xBF80, 0x3F81, 0x3B80, 0x3400, 0x0C00, 0x4000, 0xC000],
                       dtype=np.uint16)
    a = np.repeat(special, special.size)
    b = np.tile(special, special.size)
    # exponent gaps around 16 and rounding ties near 1.0
    ones = np.full(256, 0x3F80, dtype=np.uint16)
    gaps = np.array([((127 - g) << 7) | f for g in range(12, 20) for f in range(32)], dtype=np.uint16)
    a = np.concatenate([a, ones, 0x8000 | ones])
    b = np.concatenate([b, gaps, gaps])
    got = run(a, b)
    assert np.array_equal(got, reference(a, b))
    ok = (a & 0x7F80) != 0x7F80
    ok &= (b & 0x7F80) != 0x7F80
    for x, y, g in zip(a[ok][:400], b[ok][:400], got[ok][:400]):
        assert O.add_bf16(int(x), int(y)) == int(g)
