"""Hyper-connection caller oracle (src/hyper_connection.rs) pinned to the
reference's own known answers: its two unit tests
(src/hyper_connection.rs:664-679), the SHA-256 of the fixture's
deterministic hyper input (fixtures/hyper_connection/*.json, "hyper_input"),
and an independent restatement of the f32 square-sum cascade."""
import hashlib

import numpy as np
import pytest

import oracle as O

F = np.float32


def cascade_reference(values):
    """src/hyper_connection.rs:211-283 restated with numpy f32 scalars."""
    LANES, INTERLEAVE, LEVELS = 4, 4, 4
    vector_count = len(values) // LANES
    cascade = vector_count // INTERLEAVE
    ceil_log2 = 0 if cascade <= 1 else int(cascade - 1).bit_length()
    power = max(4, ceil_log2 // LEVELS)
    step = 1 << power
    mask = step - 1
    acc = [[[F(0)] * LANES for _ in range(INTERLEAVE)] for _ in range(LEVELS)]
    index = 0
    while index + step <= cascade:
        for _ in range(step):
            for r in range(INTERLEAVE):
                base = (index * INTERLEAVE + r) * LANES
                for l in range(LANES):
                    acc[0][r][l] = F(acc[0][r][l] + F(values[base + l] * values[base + l]))
            index += 1
        for level in range(1, LEVELS):
            for r in range(INTERLEAVE):
                for l in range(LANES):
                    acc[level][r][l] = F(acc[level][r][l] + acc[level - 1][r][l])
                    acc[level - 1][r][l] = F(0)
            if index & (mask << (level * power)):
                break
    while index < cascade:
        for r in range(INTERLEAVE):
            base = (index * INTERLEAVE + r) * LANES
            for l in range(LANES):
                acc[0][r][l] = F(acc[0][r][l] + F(values[base + l] * values[base + l]))
        index += 1
    for level in range(1, LEVELS):
        for r in range(INTERLEAVE):
            for l in range(LANES):
                acc[0][r][l] = F(acc[0][r][l] + acc[level][r][l])
    for vec in range(cascade * INTERLEAVE, vector_count):
        for l in range(LANES):
            v = values[vec * LANES + l]
            acc[0][0][l] = F(acc[0][0][l] + F(v * v))
    for r in range(1, INTERLEAVE):
        for l in range(LANES):
            acc[0][0][l] = F(acc[0][0][l] + acc[0][r][l])
    result = F(0)
    for v in values[vector_count * LANES:]:
        result = F(result + F(v * v))
    for l in range(LANES):
        result = F(result + acc[0][0][l])
    return result


def test_four_stream_mean_uses_sequential_reduction():
    # src/hyper_connection.rs:672-678
    assert O.four_stream_mean([1.0e8, 1.0, -1.0e8, 1.0]) == 0.25


def test_grouped_rms_is_independent_per_stream():
    # src/hyper_connection.rs:663-670 (HIDDEN = 2560 in the reference model)
    H = 2560
    ones = np.full(4 * H, O.to_bf16(1.0), dtype=np.uint16)
    out = O.grouped_rms(ones, np.zeros(4 * H, dtype=np.uint16), H)
    assert out.shape == (4 * H,) and np.all(out == O.to_bf16(1.0))


def test_hyper_input_fixture_hash():
    spec = dict(add=17, center=131, divisor=128, modulus=263, multiplier=43, sparse_stride=1)
    x = O.make_hidden(4 * 2560, spec)
    assert hashlib.sha256(x.tobytes()).hexdigest() == \
        "c489ffdc9ee671cbb4051446efe43dee9b603cefdc0e65c4d5bd464b46b54496"


@pytest.mark.parametrize("n", [3, 16, 77, 256, 2048, 2560, 4100])
def test_square_sum_cascade_matches_restatement(n):
    rng = np.random.default_rng(n)
    v = O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal(n).astype(np.float32) * 3))
    assert np.float32(O.inner_square_sum(v)) == cascade_reference([F(a) for a in v])


def test_hc_pre_and_post_shapes_and_determinism():
    L = O.HcLayer(256, 64, 4)
    post = O.synth_input(3, 5, 1024)
    m1, w1 = O.hc_pre(L, post)
    m2, w2 = O.hc_pre(L, post)
    assert m1.shape == (5, 256) and w1.shape == (5, 4)
    assert np.array_equal(m1, m2) and np.array_equal(w1, w2)
    out = O.hc_post(post, m1, w1)
    # zero injection weights leave the residual streams unchanged
    assert np.array_equal(O.hc_post(post, m1, np.zeros_like(w1)), post)
    assert out.shape == post.shape
