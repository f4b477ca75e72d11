"""GPU parity of the hyper-connection caller around the block
(src/hyper_connection.rs:412-490, src/decoder_layer.rs:451-458, 587-607)
through the C ABI: attention output post [T][4H] -> layer output [T][4H],
against the oracle (hc_pre -> block -> hc_post).  Decode widths are bit for
bit the oracle's where scores match; the prefill path is held to the block
tolerance."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)
CFG0 = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10)


def run(shape, lowrank, T, seed, min_tokens=None, max_tokens=None):
    blk = fw.MoeBlock(fw.MoeConfig(**shape, max_tokens=max_tokens or max(T, 4), layers=1))
    blk.synth_layer(0, seed, 0.02, False)
    hc = O.HcLayer(shape["hidden"], lowrank, seed + 7)
    blk.load_hc(0, lowrank, hc.norm, hc.mix_down, hc.mix_up, hc.inject)
    if min_tokens is not None:
        blk.set_prefill_min_tokens(min_tokens)
    post = O.synth_input(seed + 11, T, 4 * shape["hidden"])
    got = blk.forward_hc(0, post)
    mixed, inj = O.hc_pre(hc, post)
    bshape = O.BlockShape(**shape)
    ry, ridx, rsc = O.block(bshape, O.SynthLayer(bshape, seed, 0.02, False), mixed, threads=16)
    ref = O.hc_post(post, ry, inj)
    return got, (ref, ridx, rsc), blk


@pytest.mark.parametrize("shape,lowrank,T", [(SMALL, 64, 1), (SMALL, 64, 9), (CFG0, 320, 1), (CFG0, 320, 33)])
def test_hc_forward_matches_oracle(shape, lowrank, T):
    (out, idx, sc), (ref, ridx, rsc), _ = run(shape, lowrank, T, 21)
    assert np.array_equal(idx, ridx)
    assert int(np.abs(sc.astype(np.int32) - rsc.astype(np.int32)).max()) <= 1
    exact = np.all(sc == rsc, axis=1)
    assert np.array_equal(out[exact], ref[exact]), "bit-exact where scores match"


def test_hc_forward_prefill_path_within_tolerance():
    (out, idx, sc), (ref, ridx, rsc), _ = run(CFG0, 320, 64, 22, min_tokens=1)
    assert np.array_equal(idx, ridx)
    o, r = O.bf16_to_f32(out).astype(np.float64), O.bf16_to_f32(ref).astype(np.float64)
    # the injected part carries the block tolerance; the residual streams are exact
    assert float(np.abs(o - r).max()) <= 2e-2
    assert float(np.linalg.norm(o - r) / np.linalg.norm(r)) <= 1e-3


def test_hc_forward_repeatable_and_block_forward_unchanged():
    (out1, _, _), _, blk = run(SMALL, 64, 6, 23)
    post = O.synth_input(23 + 11, 6, 4 * SMALL["hidden"])
    out2, _, _ = blk.forward_hc(0, post)
    assert np.array_equal(out1, out2)
    # the plain block forward on the same handle still matches the oracle
    x = O.synth_input(5, 6, SMALL["hidden"])
    y, i, s = blk.forward(0, x)
    bshape = O.BlockShape(**SMALL)
    ry, ridx, rsc = O.block(bshape, O.SynthLayer(bshape, 23, 0.02, False), x)
    assert np.array_equal(i, ridx)
    exact = np.all(s == rsc, axis=1)
    assert np.array_equal(y[exact], ry[exact])


def test_hc_requires_loaded_weights():
    blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=4, layers=1))
    blk.synth_layer(0, 1, 0.02, False)
    with pytest.raises(fw.FwError):
        blk.forward_hc(0, np.zeros((2, 4 * SMALL["hidden"]), dtype=np.uint16))
    with pytest.raises(fw.FwError):
        blk.load_hc(0, 48, *(np.zeros(1, dtype=np.uint16),) * 4)  # lowrank not a multiple of 32
