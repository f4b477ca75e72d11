"""CPU checks of bench.py's parity verdicts (no GPU): the oracle's own block
output must pass both bars, one bf16 ulp in one element must fail the
decode path's bit-exact bar but pass the block tolerance, a changed expert
id must fail both, and the sampled rows must cover the hottest expert and
the last token."""
import numpy as np

import bench
import oracle as O

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=128, experts=64, top_k=4)


def _oracle_run(T, seed, zipf):
    bshape = O.BlockShape(**SMALL)
    x = O.synth_input(seed + 500, T, SMALL["hidden"])
    y, idx, sc = O.block(bshape, O.SynthLayer(bshape, seed, 0.02, zipf), x)
    return x, y, idx, sc


def test_parity_rows_accepts_the_oracle_itself():
    x, y, idx, sc = _oracle_run(12, 3, False)
    for exact in (True, False):
        r = bench.parity_rows(SMALL, 3, False, x, y, idx, sc, exact=exact)
        assert r["pass"] and r["indices_identical"] and r["max_abs"] == 0.0, r


def test_parity_rows_bars_differ_on_one_ulp():
    x, y, idx, sc = _oracle_run(12, 4, True)
    y2 = y.copy()
    y2[5, 17] = np.uint16(int(y2[5, 17]) ^ 1)  # one bf16 ulp
    exact = bench.parity_rows(SMALL, 4, True, x, y2, idx, sc, exact=True)
    tol = bench.parity_rows(SMALL, 4, True, x, y2, idx, sc, exact=False)
    assert not exact["pass"], exact
    assert tol["pass"], tol


def test_parity_rows_rejects_a_wrong_selection():
    x, y, idx, sc = _oracle_run(8, 5, False)
    idx2 = idx.copy()
    idx2[2, 0] = (idx2[2, 0] + 1) % SMALL["experts"]
    for exact in (True, False):
        r = bench.parity_rows(SMALL, 5, False, x, y, idx2, sc, exact=exact)
        assert not r["pass"] and not r["indices_identical"], r


def test_sample_rows_cover_the_hottest_expert_and_the_last_token():
    rng = np.random.default_rng(0)
    T, E, K = 300, 64, 4
    idx = np.stack([rng.choice(E, size=K, replace=False) for _ in range(T)])
    idx[::3, 0] = 7  # expert 7 is the hottest
    rows = bench.sample_rows(idx, 20, 10, 1)
    assert rows[-1] == T - 1
    assert np.sum(np.any(idx[rows] == 7, axis=1)) >= 20
    assert np.all(np.diff(rows) > 0)
