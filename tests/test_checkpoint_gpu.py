"""Loading the block and the hyper-connection weights from a safetensors
checkpoint (fw_moe_load_layer_safetensors / fw_moe_load_hc_safetensors,
through the C ABI): a sharded checkpoint with an index, and a single file,
written from the oracle's seeded weights, must give the same forward as the
same weights generated on the device, bit for bit."""
import os

import numpy as np
import pytest

import oracle as O
from st_writer import bf16_bytes, write_checkpoint, write_safetensors

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)
MLP = "model.language_model.layers.0.mlp"
HC = "model.language_model.layers.0.mlp_hyper_connection"


def layer_tensors(shape, seed):
    L = O.SynthLayer(O.BlockShape(**shape), seed)
    E, H, I, Is = (shape[k] for k in ("experts", "hidden", "intermediate", "shared_intermediate"))
    for e in range(E):
        L.expert(e)
    return {
        f"{MLP}.gate.weight": L.router.reshape(E, H),
        f"{MLP}.experts.gate_up_proj": np.concatenate([L.gate_up[e] for e in range(E)]).reshape(E, 2 * I, H),
        f"{MLP}.experts.down_proj": np.concatenate([L.down[e] for e in range(E)]).reshape(E, H, I),
        f"{MLP}.shared_expert.gate_proj.weight": L.shared_gate.reshape(Is, H),
        f"{MLP}.shared_expert.up_proj.weight": L.shared_up.reshape(Is, H),
        f"{MLP}.shared_expert.down_proj.weight": L.shared_down.reshape(H, Is),
        f"{MLP}.shared_expert_gate.weight": L.shared_gate_w.reshape(1, H),
    }


def hc_tensors(hidden, lowrank, seed):
    hc = O.HcLayer(hidden, lowrank, seed)
    HH = 4 * hidden
    return hc, {f"{HC}.hc_norm.weight": hc.norm.reshape(HH),
                f"{HC}.input_mix_weight_down.weight": hc.mix_down.reshape(lowrank, HH),
                f"{HC}.input_mix_weight_up.weight": hc.mix_up.reshape(HH, lowrank),
                f"{HC}.block_inject_weight.weight": hc.inject.reshape(4, HH)}


def test_sharded_checkpoint_equals_device_synth(tmp_path):
    t = layer_tensors(SMALL, 21)
    names = sorted(t)
    write_checkpoint(tmp_path / "ck", {"model-00001-of-00002.safetensors": {n: t[n] for n in names[:3]},
                                      "model-00002-of-00002.safetensors": {n: t[n] for n in names[3:]}})
    blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=8, layers=2))
    blk.synth_layer(0, 21)
    blk.load_layer_safetensors(1, str(tmp_path / "ck"), MLP)
    x = O.synth_input(77, 8, SMALL["hidden"])
    for u, v in zip(blk.forward(0, x), blk.forward(1, x)):
        assert np.array_equal(u, v)


def test_single_file_and_hyper_connection(tmp_path):
    t = layer_tensors(SMALL, 22)
    hc, ht = hc_tensors(SMALL["hidden"], 64, 5)
    f = tmp_path / "model.safetensors"
    write_safetensors(f, {n: ("BF16", a.shape, bf16_bytes(a)) for n, a in {**t, **ht}.items()})
    blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=6, layers=2))
    blk.synth_layer(0, 22)
    blk.load_hc(0, 64, hc.norm, hc.mix_down, hc.mix_up, hc.inject)
    blk.load_layer_safetensors(1, str(f), MLP)
    blk.load_hc_safetensors(1, str(f), HC)
    post = O.synth_input(3, 6, 4 * SMALL["hidden"])
    for u, v in zip(blk.forward_hc(0, post), blk.forward_hc(1, post)):
        assert np.array_equal(u, v)


def test_shape_and_name_mismatches_fail_closed(tmp_path):
    t = layer_tensors(SMALL, 23)
    f = tmp_path / "model.safetensors"
    write_safetensors(f, {n: ("BF16", a.shape, bf16_bytes(a)) for n, a in t.items()})
    wrong = dict(SMALL, intermediate=64)
    blk = fw.MoeBlock(fw.MoeConfig(**wrong, max_tokens=4, layers=1))
    with pytest.raises(fw.FwError) as e:
        blk.load_layer_safetensors(0, str(f), MLP)
    assert "gate_up_proj" in str(e.value)
    blk2 = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=4, layers=1))
    with pytest.raises(fw.FwError) as e:
        blk2.load_layer_safetensors(0, str(f), "model.language_model.layers.7.mlp")
    assert "absent" in str(e.value)
    # an index naming a shard outside the directory
    d = tmp_path / "ck"
    write_checkpoint(d, {"a.safetensors": t})
    idx = (d / "model.safetensors.index.json").read_text().replace('"a.safetensors"', '"../a.safetensors"')
    (d / "model.safetensors.index.json").write_text(idx)
    with pytest.raises(fw.FwError) as e:
        blk2.load_layer_safetensors(0, str(d), MLP)
    assert "unbound checkpoint shard" in str(e.value)
    # the handle stays usable
    blk2.load_layer_safetensors(0, str(f), MLP)
    y, _, _ = blk2.forward(0, O.synth_input(1, 4, SMALL["hidden"]))
    assert np.all(np.isfinite(O.bf16_to_f32(y)))
