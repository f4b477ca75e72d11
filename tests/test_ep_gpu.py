"""Expert parallelism on 2, 4 and 8 GPUs through the C ABI: each rank holds
1/world of the experts (fw_moe_ep_init), brings its own tokens, and must
return the single-GPU result for them: on the decode path the oracle's block
output, bit for bit where scores match, and the same selection everywhere;
on the prefill path the same selection and the block tolerance.  Both
transports are covered: NVLink peer memory (the default) and NCCL.  A case
is skipped when fewer GPUs than its world are visible.

The failure case stops one rank between forwards (it stays alive, takes no
part in the next forward, and exits only after the others are done): the
others' next forward must fail closed within the wait limit, with no fault
and no hang.  NCCL's NVLink multicast (NVLS) is off in every rank.
"""
import os
import tempfile
import time
from datetime import timedelta

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)
CFG0 = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10)
# Benchmark config 4's block.
CFG4 = dict(hidden=3072, intermediate=768, shared_intermediate=768, experts=512, top_k=10)

P2P, NCCL = 0, 1
PATH_DECODE, PATH_PREFILL = 1, 2  # fw_moe_last_path


def _rendezvous() -> str:
    """A file-based rendezvous (no port to collide with another process)."""
    d = tempfile.mkdtemp(prefix="fw_ep_")
    return "file://" + os.path.join(d, "store")


def _setup(rank, world, store):
    import torch.distributed as dist

    # No NVLink multicast objects in a test that may stop a rank early.
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    # a rank that fails ends the other's collectives within a minute
    dist.init_process_group("gloo", init_method=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    return dist


def _rank_main(rank, world, store, shape, t_local, layers, zipf, q, min_tokens, transport, hc_lowrank):
    import firewing_b200 as fw

    dist = _setup(rank, world, store)
    try:
        uid = [fw.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        cfg = fw.MoeConfig(**shape, max_tokens=t_local, layers=layers)
        blk = fw.MoeBlock(cfg, device=rank)
        blk.ep_init(rank, world, uid[0], transport)
        if min_tokens is not None:
            blk.set_prefill_min_tokens(min_tokens)
        hcs = []
        for l in range(layers):
            blk.synth_layer(l, 40 + l, 0.02, zipf)
            if hc_lowrank:
                hc = O.HcLayer(shape["hidden"], hc_lowrank, 60 + l)
                blk.load_hc(l, hc_lowrank, hc.norm, hc.mix_down, hc.mix_up, hc.inject)
                hcs.append(hc)
        width = 4 * shape["hidden"] if hc_lowrank else shape["hidden"]
        results = []
        for l in range(layers):
            x_all = O.synth_input(900 + l, world * t_local, width)
            x = x_all[rank * t_local:(rank + 1) * t_local].copy()
            fwd = blk.forward_hc if hc_lowrank else blk.forward
            y1, i1, s1 = fwd(l, x)
            path = blk.last_path()
            y2, i2, s2 = fwd(l, x)  # repeatable
            results.append((l, x_all, y1, i1, s1, bool(np.array_equal(y1, y2) and np.array_equal(i1, i2)), path))
        blk.close()
        gathered = [None] * world
        dist.all_gather_object(gathered, [(l, y, i, s, rep) for (l, _, y, i, s, rep, _) in results])
        if rank == 0:
            bshape = O.BlockShape(**shape)
            report = []
            for l in range(layers):
                x_all = results[l][1]
                y = np.concatenate([gathered[r][l][1] for r in range(world)])
                i = np.concatenate([gathered[r][l][2] for r in range(world)])
                s = np.concatenate([gathered[r][l][3] for r in range(world)])
                rep = all(gathered[r][l][4] for r in range(world))
                layer = O.SynthLayer(bshape, 40 + l, 0.02, zipf)
                if hc_lowrank:
                    mixed, inj = O.hc_pre(hcs[l], x_all)
                    ry, ridx, rsc = O.block(bshape, layer, mixed, threads=os.cpu_count() or 1)
                    ry = O.hc_post(x_all, ry, inj)
                else:
                    ry, ridx, rsc = O.block(bshape, layer, x_all, threads=os.cpu_count() or 1)
                exact = np.all(s == rsc, axis=1)
                yf, rf = O.bf16_to_f32(y).astype(np.float64), O.bf16_to_f32(ry).astype(np.float64)
                report.append(dict(path=results[l][6], idx=bool(np.array_equal(i, ridx)),
                                   score_ulp=int(np.abs(s.astype(np.int32) - rsc.astype(np.int32)).max()),
                                   exact_tokens_equal=bool(np.array_equal(y[exact], ry[exact])),
                                   n_exact=int(exact.sum()), repeat=rep,
                                   max_abs=float(np.abs(yf - rf).max()),
                                   rel_l2=float(np.linalg.norm(yf - rf) / max(np.linalg.norm(rf), 1e-30))))
            q.put(report)
    finally:
        dist.destroy_process_group()


def _spawn(target, world, args, timeout=300):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = _rendezvous()
    procs = [ctx.Process(target=target, args=(r, world, store, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(timeout=30)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return q.get(timeout=5)


def _run(shape, t_local, layers, zipf, min_tokens=None, world=2, transport=P2P, hc_lowrank=0):
    return _spawn(_rank_entry, world, (shape, t_local, layers, zipf, min_tokens, transport, hc_lowrank))


def _rank_entry(rank, world, store, shape, t_local, layers, zipf, min_tokens, transport, hc_lowrank, q):
    _rank_main(rank, world, store, shape, t_local, layers, zipf, q, min_tokens, transport, hc_lowrank)


def _decode_ok(r):
    return (r["path"] == PATH_DECODE and r["idx"] and r["score_ulp"] <= 1 and r["exact_tokens_equal"]
            and r["repeat"])


def _prefill_ok(r):
    return (r["path"] == PATH_PREFILL and r["idx"] and r["score_ulp"] <= 1 and r["repeat"]
            and r["max_abs"] <= 2e-2 and r["rel_l2"] <= 1e-3)


@pytest.mark.parametrize("transport", [P2P, NCCL])
@pytest.mark.parametrize("t_local,zipf", [(1, False), (7, False), (32, True)])
def test_ep_two_gpus_small_shape(t_local, zipf, transport):
    for r in _run(SMALL, t_local, 2, zipf, transport=transport):
        assert _decode_ok(r), r


@pytest.mark.parametrize("transport", [P2P, NCCL])
def test_ep_two_gpus_config0_shape(transport):
    for r in _run(CFG0, 32, 1, False, transport=transport):
        assert _decode_ok(r), r


# Prefill path under expert parallelism (tensor-core GEMMs): the block
# tolerance of the north star, identical selection.
@pytest.mark.parametrize("transport", [P2P, NCCL])
@pytest.mark.parametrize("shape,t_local,min_tokens,zipf", [(SMALL, 300, None, True), (SMALL, 40, 1, False),
                                                          (CFG4, 160, 1, True)])
def test_ep_two_gpus_prefill(shape, t_local, min_tokens, zipf, transport):
    for r in _run(shape, t_local, 1, zipf, min_tokens, transport=transport):
        assert _prefill_ok(r), r


# Config 0's block at 2, 4 and 8 GPUs on both paths (peer-memory transport).
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_config0_decode(world):
    # 16 tokens per rank, the decode path pinned (a set threshold counts
    # every rank's tokens too)
    for r in _run(CFG0, 16, 2, False, min_tokens=1 << 20, world=world):
        assert _decode_ok(r), r


# The default path threshold (96 tokens) counts every rank's tokens: 2 x 48
# take the tensor-core path, 2 x 47 the decode path.
@pytest.mark.parametrize("t_local", [47, 48])
def test_ep_default_path_counts_all_ranks(t_local):
    for r in _run(CFG0, t_local, 1, False):
        assert (_prefill_ok(r) if t_local == 48 else _decode_ok(r)), r


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_config0_prefill(world):
    for r in _run(CFG0, 64, 1, True, min_tokens=1, world=world):
        assert _prefill_ok(r), r


# The hyper-connection caller around an expert-parallel block
# (src/decoder_layer.rs:451-458, 587-607): per-token stages on each rank.
@pytest.mark.parametrize("min_tokens", [None, 1])
def test_ep_two_gpus_hyper_connection(min_tokens):
    for r in _run(CFG0, 8, 1, False, min_tokens=min_tokens, hc_lowrank=320):
        assert (_decode_ok(r) if min_tokens is None else _prefill_ok(r)), r


# ---- failing closed ----------------------------------------------------------

def _stop_main(rank, world, store, transport, wait_s, q):
    import firewing_b200 as fw

    dist = _setup(rank, world, store)
    try:
        uid = [fw.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        blk = fw.MoeBlock(fw.MoeConfig(**SMALL, max_tokens=8, layers=1), device=rank)
        blk.ep_init(rank, world, uid[0], transport)
        blk.set_wait_limit(wait_s)
        blk.synth_layer(0, 3, 0.02, False)
        x = O.synth_input(100 + rank, 8, SMALL["hidden"])
        blk.forward(0, x)  # a complete forward on every rank
        dist.barrier()
        if rank == 1:
            # This rank stops between forwards: it keeps its process (and its
            # window) but takes no part in the next forward; it leaves only
            # after rank 0 has finished.
            dist.barrier()
            blk.close()
            return
        t0 = time.monotonic()
        code = None
        try:
            blk.forward(0, x)
        except fw.FwError as e:
            code = e.code
        elapsed = time.monotonic() - t0
        blk.close()
        q.put({"code": code, "elapsed": elapsed})
        dist.barrier()
    finally:
        dist.destroy_process_group()


# Over peer memory the dispatch's bounded wait on the silent peer's flag
# runs out and every later kernel of the forward skips its work.
def test_ep_peer_stops_between_forwards_fails_closed():
    import firewing_b200 as fw

    wait_s = 1.0
    r = _spawn(_stop_main, 2, (P2P, wait_s), timeout=180)
    assert r["code"] == fw.FW_ETIMEOUT, r
    assert r["elapsed"] < 10 * wait_s, r
