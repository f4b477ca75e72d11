"""Expert parallelism, host side, on CPU: two gloo ranks run the decomposition
that fw_moe_ep_init switches the library to, with the oracle's primitives in
place of the kernels, and must reproduce the single-device oracle block bit
for bit.

Per rank: router and route on its own tokens; all-gather of token rows, top-k
ids and route weights; its experts (ep_expert_range) over every gathered
pair (ep_held_experts: interleaved placement); the weighted rows returned to
each token's owner in the receive layout of ep_combine_row; the owner's
ascending-expert-id sum plus its shared expert.
"""
import os
import tempfile
from datetime import timedelta

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import firewing_b200 as fw  # noqa: E402

SHAPE = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)


def _rendezvous() -> str:
    """A file-based rendezvous (no port to collide with another process)."""
    d = tempfile.mkdtemp(prefix="fw_ep_")
    return "file://" + os.path.join(d, "store")


def _bf16_add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return O.f32_to_bf16(O.bf16_to_f32(a) + O.bf16_to_f32(b))


def _bf16_mul(a: np.ndarray, s: np.ndarray) -> np.ndarray:
    return O.f32_to_bf16(O.bf16_to_f32(a) * O.bf16_to_f32(s))


def _gather(arr: np.ndarray, world: int) -> np.ndarray:
    # gloo moves 32-bit integers; bf16 bit patterns ride in int32
    t = torch.from_numpy(np.ascontiguousarray(arr).astype(np.int32))
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return torch.cat(out).numpy().astype(arr.dtype)


def _rank_main(rank: int, world: int, store: str, seed: int, t_local: int, zipf: bool, q) -> None:
    dist.init_process_group("gloo", init_method=store, rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        shape = O.BlockShape(**SHAPE)
        H, I, Is, E, K = (SHAPE[k] for k in ("hidden", "intermediate", "shared_intermediate", "experts",
                                              "top_k"))
        layer = O.SynthLayer(shape, seed, 0.02, zipf)
        x_all_ref = O.synth_input(seed + 500, world * t_local, H)
        x = x_all_ref[rank * t_local:(rank + 1) * t_local].copy()
        # 1. router + route on this rank's tokens
        idx, score, _ = O.router(shape, layer, x)
        # 2. dispatch: every rank's rows, ids and weights
        x_all = _gather(x, world)
        idx_all = _gather(idx, world)
        score_all = _gather(score, world)
        # 3. this rank's experts over every gathered pair: weighted rows in
        #    the [global token][K][H] send layout
        held = set(fw.ep_held_experts(E, world, rank))
        send = np.zeros((world * t_local * K, H), dtype=np.uint16)
        for t in range(world * t_local):
            for k in range(K):
                e = int(idx_all[t, k])
                if e not in held:
                    continue
                gu, dn = layer.expert(e)
                g = O.linear_bf16(gu[: I * H], x_all[t], I, H)
                u = O.linear_bf16(gu[I * H:], x_all[t], I, H)
                a = O.swiglu_bf16(g, u)
                d = O.linear_bf16(dn, a, H, I)
                send[t * K + k] = _bf16_mul(d, np.full(H, score_all[t, k], dtype=np.uint16))
        # 4. combine exchange: block d of every rank's send buffer goes to
        #    rank d (gathered whole here; the library sends only block d)
        sends = _gather(send, world).reshape(world, world * t_local * K, H)
        blk = slice(rank * t_local * K, (rank + 1) * t_local * K)
        recv = np.concatenate([sends[src][blk] for src in range(world)])
        # 5. owner: ascending expert id sum, then the shared expert
        y = np.empty((t_local, H), dtype=np.uint16)
        for tl in range(t_local):
            acc = np.zeros(H, dtype=np.uint16)
            for k in np.argsort(idx[tl], kind="stable"):
                row = fw.ep_combine_row(int(idx[tl, k]), tl, int(k), t_local, K, world)
                acc = _bf16_add(acc, recv[row])
            sg = O.linear_bf16(layer.shared_gate, x[tl], Is, H)
            su = O.linear_bf16(layer.shared_up, x[tl], Is, H)
            sd = O.linear_bf16(layer.shared_down, O.swiglu_bf16(sg, su), H, Is)
            gate = O.sigmoid_bf16(int(O.linear_bf16(layer.shared_gate_w, x[tl], 1, H)[0]))
            y[tl] = _bf16_add(acc, _bf16_mul(sd, np.full(H, gate, dtype=np.uint16)))
        y_all = _gather(y, world)
        idx_g = _gather(idx, world)
        if rank == 0:
            ry, ridx, _ = O.block(shape, O.SynthLayer(shape, seed, 0.02, zipf), x_all_ref)
            q.put((bool(np.array_equal(idx_g, ridx)), bool(np.array_equal(y_all, ry)),
                   int((y_all != ry).any(axis=1).sum())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("zipf", [False, True])
def test_ep_decomposition_matches_single_device_oracle(zipf):
    world, t_local = 2, 6
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = _rendezvous()
    procs = [ctx.Process(target=_rank_main, args=(r, world, store, 31, t_local, zipf, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same_idx, same_y, bad_tokens = q.get(timeout=5)
    assert same_idx
    assert same_y, f"{bad_tokens} tokens differ"


def test_ep_host_helpers():
    assert fw.ep_held_experts(512, 8, 3)[:3] == [3, 11, 19] and len(fw.ep_held_experts(512, 8, 3)) == 64
    with pytest.raises(ValueError):
        fw.ep_held_experts(512, 3, 0)
    # expert 70 lives on rank 70 % 8 = 6: its rows arrive in block 6
    assert fw.ep_owner(70, 8) == 6
    assert fw.ep_combine_row(70, 5, 2, 32, 10, 8) == (6 * 32 + 5) * 10 + 2
    # one rank: the single-GPU layout t*K + k
    assert fw.ep_combine_row(511, 7, 9, 64, 10, 1) == 7 * 10 + 9
