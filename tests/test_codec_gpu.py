"""Loading experts from a compressed container (fw_moe_load_expert_container)
and one at a time (fw_moe_load_expert), through the C ABI: the block must
then equal the oracle with those experts replaced, bit for bit at decode
widths."""
import numpy as np
import pytest

import oracle as O
from codec_writer import expert_source, write_container

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)


def replacement(e):
    """Expert e's weights from another seed."""
    other = O.SynthLayer(O.BlockShape(**SMALL), 99)
    return other.expert(e)


def test_container_and_single_expert_loads_match_oracle(tmp_path):
    # replace the experts the input actually selects (and one it does not)
    bshape = O.BlockShape(**SMALL)
    x = O.synth_input(7, 8, SMALL["hidden"])
    ref_layer = O.SynthLayer(bshape, 21)
    idx0, _, _ = O.router(bshape, ref_layer, x)
    chosen = sorted(set(int(v) for v in idx0.ravel()))[:6] + [63]
    for e in chosen:
        ref_layer.gate_up[e], ref_layer.down[e] = replacement(e)
    ry, ridx, rsc = O.block(bshape, ref_layer, x)

    m = write_container(tmp_path, {(5, e): expert_source(*replacement(e)) for e in chosen})
    blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=8, layers=2))
    blk.synth_layer(0, 21)
    blk.synth_layer(1, 21)
    assert blk.load_expert_container(0, m, 5, verify=True) == len(chosen)
    for e in chosen:
        blk.load_expert(1, e, *replacement(e))
    for layer in (0, 1):
        y, idx, sc = blk.forward(layer, x)
        assert np.array_equal(idx, ridx)
        exact = np.all(sc == rsc, axis=1)
        assert exact.sum() >= 6 and np.array_equal(y[exact], ry[exact])
    # a container layer with no records loads nothing; bad expert ids fail closed
    assert blk.load_expert_container(0, m, 4) == 0
    with pytest.raises(fw.FwError):
        blk.load_expert(0, 64, *replacement(0))
