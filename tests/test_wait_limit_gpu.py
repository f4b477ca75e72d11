"""Bounded device waits fail closed: a test hook (fw_moe_test_stall) makes
the expert kernel's wait for its gate/up units unreachable, so that wait
runs out after the handle's wait limit (fw_moe_set_wait_limit).  The forward
must report FW_ETIMEOUT promptly, the device must stay usable, and the next
forward on the same handle must be correct again.  Nothing here faults or
hangs the GPU: the wait gives up, records the status and the kernel exits.
"""
import time

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)


@pytest.mark.parametrize("T", [2, 8])  # the small-width kernel and the 8-token-pass kernel
def test_expert_wait_runs_out_and_handle_recovers(T):
    blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=8, layers=1))
    blk.synth_layer(0, 9, 0.02, False)
    x = O.synth_input(10, T, SMALL["hidden"])
    good = blk.forward(0, x)
    blk.set_wait_limit(0.05)
    blk.test_stall()
    t0 = time.monotonic()
    with pytest.raises(fw.FwError) as e:
        blk.forward(0, x)
    assert e.value.code == fw.FW_ETIMEOUT
    assert time.monotonic() - t0 < 5.0
    again = blk.forward(0, x)
    assert all(np.array_equal(u, v) for u, v in zip(good, again))
    bshape = O.BlockShape(**SMALL)
    ry, ridx, _ = O.block(bshape, O.SynthLayer(bshape, 9), x)
    assert np.array_equal(again[1], ridx)


def test_wait_limit_bounds_are_checked():
    blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=4, layers=1))
    with pytest.raises(fw.FwError):
        blk.set_wait_limit(0.0)
    with pytest.raises(fw.FwError):
        blk.set_wait_limit(120.0)
