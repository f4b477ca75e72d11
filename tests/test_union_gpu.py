"""Expert-union accounting of a forward (fw_moe_last_union): the distinct
routed experts a forward streamed and the bytes it read, which a caller
combines with its accepted tokens into the reference's A / U figure for
speculative verification (docs/ARCHITECTURE.md:93-96).  Checked against the
forward's own top-k ids on the decode and the prefill path."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)


def expected_bytes(shape, u):
    H, I, Is, E = (shape[k] for k in ("hidden", "intermediate", "shared_intermediate", "experts"))
    return 2 * (E * H + H + 3 * H * Is + u * 3 * H * I)


@pytest.mark.parametrize("T,min_tokens", [(1, None), (4, None), (64, None), (300, None), (40, 1)])
def test_union_matches_selection(T, min_tokens):
    blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=max(T, 8), layers=1))
    blk.synth_layer(0, 31, 0.02, True)
    if min_tokens is not None:
        blk.set_prefill_min_tokens(min_tokens)
    with pytest.raises(fw.FwError):
        blk.last_union()
    _, idx, _ = blk.forward(0, O.synth_input(5, T, SMALL["hidden"]))
    u = blk.last_union()
    distinct = len(np.unique(idx))
    assert u["distinct_experts"] == distinct
    assert u["weight_bytes"] == expected_bytes(SMALL, distinct)
    # verify width T: each distinct expert streamed once for all T tokens
    assert distinct <= min(SMALL["experts"], T * SMALL["top_k"])
