"""Expert parallelism on 2, 4 and 8 GPUs through the C ABI: each rank holds
1/world of the experts (fw_moe_ep_init), brings its own tokens, and must
return the single-GPU result for them: on the decode path the oracle's block
output, bit for bit where scores match, and the same selection everywhere;
on the prefill path the same selection and the block tolerance.  A case is
skipped when fewer GPUs than its world are visible.
"""
import os
import tempfile
from datetime import timedelta

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)
CFG0 = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10)


def _rendezvous() -> str:
    """A file-based rendezvous (no port to collide with another process)."""
    d = tempfile.mkdtemp(prefix="fw_ep_")
    return "file://" + os.path.join(d, "store")


def _rank_main(rank, world, store, shape, t_local, layers, zipf, q, min_tokens=None):
    import torch.distributed as dist

    import firewing_b200 as fw

    # No NVLink multicast objects in a test that may stop a rank early.
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    # a rank that fails ends the other's collectives within a minute
    dist.init_process_group("gloo", init_method=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        uid = [fw.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        cfg = fw.MoeConfig(**shape, max_tokens=t_local, layers=layers)
        blk = fw.MoeBlock(cfg, device=rank)
        blk.ep_init(rank, world, uid[0])
        if min_tokens is not None:
            blk.set_prefill_min_tokens(min_tokens)
        for l in range(layers):
            blk.synth_layer(l, 40 + l, 0.02, zipf)
        results = []
        for l in range(layers):
            x_all = O.synth_input(900 + l, world * t_local, shape["hidden"])
            x = x_all[rank * t_local:(rank + 1) * t_local].copy()
            y1, i1, s1 = blk.forward(l, x)
            y2, i2, s2 = blk.forward(l, x)  # repeatable
            results.append((l, x_all, y1, i1, s1, bool(np.array_equal(y1, y2) and np.array_equal(i1, i2))))
        blk.close()
        gathered = [None] * world
        dist.all_gather_object(gathered, [(l, y, i, s, rep) for (l, _, y, i, s, rep) in results])
        if rank == 0:
            bshape = O.BlockShape(**shape)
            report = []
            for l in range(layers):
                x_all = results[l][1]
                y = np.concatenate([gathered[r][l][1] for r in range(world)])
                i = np.concatenate([gathered[r][l][2] for r in range(world)])
                s = np.concatenate([gathered[r][l][3] for r in range(world)])
                rep = all(gathered[r][l][4] for r in range(world))
                ry, ridx, rsc = O.block(bshape, O.SynthLayer(bshape, 40 + l, 0.02, zipf), x_all,
                                        threads=os.cpu_count() or 1)
                exact = np.all(s == rsc, axis=1)
                yf, rf = O.bf16_to_f32(y).astype(np.float64), O.bf16_to_f32(ry).astype(np.float64)
                report.append(dict(idx=bool(np.array_equal(i, ridx)),
                                   score_ulp=int(np.abs(s.astype(np.int32) - rsc.astype(np.int32)).max()),
                                   exact_tokens_equal=bool(np.array_equal(y[exact], ry[exact])),
                                   n_exact=int(exact.sum()), repeat=rep,
                                   max_abs=float(np.abs(yf - rf).max()),
                                   rel_l2=float(np.linalg.norm(yf - rf) / max(np.linalg.norm(rf), 1e-30))))
            q.put(report)
    finally:
        dist.destroy_process_group()


def _run(shape, t_local, layers, zipf, min_tokens=None, world=2):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = _rendezvous()
    procs = [ctx.Process(target=_rank_main, args=(r, world, store, shape, t_local, layers, zipf, q, min_tokens))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(timeout=30)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return q.get(timeout=5)


@pytest.mark.parametrize("t_local,zipf", [(1, False), (7, False), (32, True)])
def test_ep_two_gpus_small_shape(t_local, zipf):
    for r in _run(SMALL, t_local, 2, zipf):
        assert r["idx"] and r["score_ulp"] <= 1 and r["exact_tokens_equal"] and r["repeat"], r


def test_ep_two_gpus_config0_shape():
    for r in _run(CFG0, 32, 1, False):
        assert r["idx"] and r["score_ulp"] <= 1 and r["exact_tokens_equal"] and r["repeat"], r


# Prefill path under expert parallelism (tensor-core GEMMs, row-sized
# exchange): the block tolerance of the north star, identical selection.
CFG4 = dict(hidden=3072, intermediate=768, shared_intermediate=768, experts=512, top_k=10)


@pytest.mark.parametrize("shape,t_local,min_tokens,zipf", [(SMALL, 300, None, True), (SMALL, 40, 1, False),
                                                          (CFG4, 160, 1, True)])
def test_ep_two_gpus_prefill(shape, t_local, min_tokens, zipf):
    for r in _run(shape, t_local, 1, zipf, min_tokens):
        assert r["idx"] and r["score_ulp"] <= 1 and r["repeat"], r
        assert r["max_abs"] <= 2e-2 and r["rel_l2"] <= 1e-3, r


# Config 0's block at 2, 4 and 8 GPUs on both paths.
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_config0_decode(world):
    for r in _run(CFG0, 16, 2, False, world=world):
        assert r["idx"] and r["score_ulp"] <= 1 and r["exact_tokens_equal"] and r["repeat"], r


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_config0_prefill(world):
    for r in _run(CFG0, 64, 1, True, min_tokens=1, world=world):
        assert r["idx"] and r["score_ulp"] <= 1 and r["repeat"], r
        assert r["max_abs"] <= 2e-2 and r["rel_l2"] <= 1e-3, r
