#!/usr/bin/env python
"""Sparse-MoE block benchmark (tokens/s + roofline) on B200.

Default workload = benchmark config 1: a 24-layer stack of the config-0 block
(H=2048, 512 experts, top-10, I = Is = 512, bf16 weights ~N(0,0.02) from
seeds 1..24, inputs bf16 N(0,1) RMS-normalised), decode at T=64 tokens per
layer (T=4 is reported alongside).  A step = every layer of the stack over
its T tokens, layers in order on one stream.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on stdout (rank 0).  --impl reference times the CPU oracle (a
line-for-line C restatement of the reference's CPU block path; the Rust
crate itself cannot build on Linux) on the box's host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "cfg1": dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10,
                 layers=24, tokens=64, zipf=False,
                 name="cfg1: 24-layer stack of the config-0 block, decode"),
}
# Reported alongside at N > 1 (not the headline): benchmark config 3, expert
# parallelism over the N GPUs.
EP = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10,
          tokens=256, layers=24, layers_8=48,
          name="cfg3: {layers}-layer stack of the config-0 block, EP over {world} GPUs ({per} experts "
               "per GPU), decode T=256 per layer, uniform routing")
# Reported alongside (not the headline): benchmark config 4, the larger block
# at prefill width, 12 layers; one GPU at N = 1, expert-parallel at N > 1.
CFG4 = dict(hidden=3072, intermediate=768, shared_intermediate=768, experts=512, top_k=10,
            tokens=8192, layers=12, zipf=True,
            name="cfg4: 12-layer stack, H=3072, I=Is=768, Zipf-biased router, prefill T=8192 per GPU")
# Reported alongside (not the headline): benchmark config 2, one block at
# prefill width with the Zipf-biased router, on the tensor-core path.
PREFILL = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10,
               tokens=8192, zipf=True, seed=1,
               name="cfg2: one config-0 block, prefill T=8192, Zipf-biased router")
METRIC = "MoE-block tokens/s (token-layers per second through the block)"
UNIT = "tokens/s"


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def layer_seed(layer: int) -> int:
    return layer + 1  # config 1: per-layer weights from seeds 1..24


def input_seed(rank: int, layer: int) -> int:
    return 1_000_000 + 1000 * rank + layer


def algorithmic_bytes(w: dict, T: int, unique: int) -> int:
    """Bytes a layer must move at minimum: the distinct experts' weights,
    router, shared expert, shared gate vector, inputs and outputs."""
    H, I, Is, E = w["hidden"], w["intermediate"], w["shared_intermediate"], w["experts"]
    return unique * 3 * H * I * 2 + E * H * 2 + 3 * H * Is * 2 + H * 2 + T * H * 2 * 2


def experts_kernel_bytes(w: dict, T: int, unique: int, pairs: int) -> int:
    """Algorithmic bytes of the expert kernel: the distinct experts' gate_up
    and down slices, the shared expert, activations in, SwiGLU rows out and
    back in, weighted rows out."""
    H, I, Is = w["hidden"], w["intermediate"], w["shared_intermediate"]
    weights = unique * 3 * I * H * 2 + 3 * Is * H * 2
    acts = (pairs + T) * H * 2 + 2 * (pairs * I + T * Is) * 2 + (pairs + T) * H * 2
    return weights + acts


# ---------------------------------------------------------------------------
# clocks during the timed region

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.device), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        time.sleep(0.2)
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        for line in (self.out or "").splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                  "sw_power_cap"), f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = sorted(sm)[len(sm) // 2:] or sm  # upper half: samples under load
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU side (oracle = line-for-line C restatement of the reference CPU path)

def cpu_run(w: dict, layers, tokens: int, threads: int, rank: int = 0):
    """Prepare host weights for `layers` and return a callable timing one
    pass of the oracle over those layers' first `tokens` tokens."""
    import oracle as O
    from concurrent.futures import ThreadPoolExecutor

    shape = O.BlockShape(w["hidden"], w["intermediate"], w["shared_intermediate"], w["experts"],
                         w["top_k"])
    prepared = []
    for l in layers:
        L = O.SynthLayer(shape, layer_seed(l), 0.02, w["zipf"])
        x = O.synth_input(input_seed(rank, l), tokens, w["hidden"])
        idx, _, _ = O.router(shape, L, x)
        with ThreadPoolExecutor(max(1, threads)) as ex:
            list(ex.map(L.expert, sorted(set(idx.ravel().tolist()))))
        prepared.append((L, x))

    def one_pass():
        outs = []
        for L, x in prepared:
            outs.append(O.block_resident(shape, L, x, threads=threads))
        return outs

    return one_pass


def cpu_baseline(w: dict, threads: int, budget_s: float = 10.0, rank: int = 0) -> dict:
    sample_layers = [0, 1]
    tokens = w["tokens"]
    one_pass = cpu_run(w, sample_layers, tokens, threads, rank)
    one_pass()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        one_pass()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    tl = n * len(sample_layers) * tokens
    return {"value": tl / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"layers {sample_layers} x {tokens} tokens of the same workload, "
                       f"{n} passes, {el:.1f} s; token-layers/s with {threads} threads "
                       "(tokens spread over threads)")}


def run_reference(args, w: dict, rank: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    tokens = w["tokens"]
    one_pass = cpu_run(w, [0], tokens, threads, rank)
    for _ in range(args.warmup):
        one_pass()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_pass()
    el = time.perf_counter() - t0
    value = args.steps * tokens / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": w["name"], "layers_per_step": 1, "tokens": tokens,
                   "hidden": w["hidden"], "experts": w["experts"], "top_k": w["top_k"],
                   "intermediate": w["intermediate"]},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"layer 0 x {tokens} tokens per step (bounded sample of the "
                                   "24-layer workload), tokens spread over host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side

def run_ours(args, w: dict, rank: int, world: int, local_rank: int) -> None:
    import torch

    import firewing_b200 as fw
    from firewing_b200 import synth

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
    H, K = w["hidden"], w["top_k"]
    L = args.layers or w["layers"]
    T = args.tokens or w["tokens"]
    cfg = fw.MoeConfig(w["hidden"], w["intermediate"], w["shared_intermediate"], w["experts"], K,
                       max_tokens=max(T, 4), layers=L)
    blk = fw.MoeBlock(cfg, device=local_rank)
    for l in range(L):
        blk.synth_layer(l, layer_seed(l), 0.02, w["zipf"])
    stream = torch.cuda.Stream()

    def device_inputs(tokens):
        xs = np.stack([synth.synth_input(input_seed(rank, l), tokens, H) for l in range(L)])
        return torch.from_numpy(xs.view(np.int16)).cuda()

    def make_bufs(tokens):
        return (device_inputs(tokens),
                torch.empty((L, tokens, H), dtype=torch.int16, device="cuda"),
                torch.empty((L, tokens, K), dtype=torch.int32, device="cuda"),
                torch.empty((L, tokens, K), dtype=torch.int16, device="cuda"))

    def step(tokens, bufs):
        x, y, idx, sc = bufs
        for l in range(L):
            blk.forward_async(l, x[l], tokens, y[l], idx[l], sc[l], stream=stream)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(tokens, bufs, steps, warmup, sampler=None):
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                step(tokens, bufs)
        blk.sync(stream)
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx = sampler if sampler is not None else _Null()
        with ctx:
            e0.record(stream)
            for _ in range(steps):
                step(tokens, bufs)
            e1.record(stream)
            e1.synchronize()
        blk.sync(stream)
        barrier()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / 1e3)

    bufs = make_bufs(T)
    sampler = ClockSampler(local_rank)
    el = timed(T, bufs, args.steps, args.warmup, sampler)
    clocks = sampler.summary()
    if args.minimal:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": world * T * L * args.steps / el,
                              "unit": UNIT, "minimal": True, "layers": L, "tokens": T}))
        blk.close()
        return
    value = world * T * L * args.steps / el
    # routing statistics of the run itself (distinct experts per layer)
    idx_host = bufs[2].cpu().numpy()
    unique = [len(np.unique(idx_host[l])) for l in range(L)]
    step_bytes = sum(algorithmic_bytes(w, T, u) for u in unique)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        hbm_peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except Exception:
        hbm_peak, peak_src = 6650.0, "fallback"

    # dominant kernel: per-stage CUDA events in a separate pass after the
    # timed region (events between kernels serialise them)
    def stage_profile(tokens, bufs_, uniq, steps=3):
        blk.profile(True)
        tot = {s_: 0.0 for s_ in fw.MoeBlock.STAGES}
        kb = 0
        xx, yy, ii, ss = bufs_
        with torch.cuda.stream(stream):
            for _ in range(steps):
                for l in range(L):
                    blk.forward_async(l, xx[l], tokens, yy[l], ii[l], ss[l], stream=stream)
                    for k_, v_ in blk.profile_read().items():
                        tot[k_] += v_
                    kb += experts_kernel_bytes(w, tokens, uniq[l], tokens * K)
        blk.profile(False)
        return tot, kb, steps * L

    stage_tot, up_bytes, prof_n = stage_profile(T, bufs, unique)
    up_s = stage_tot["experts"] / 1e3
    up_gbs = up_bytes / up_s / 1e9
    traffic = None
    prof_path = os.path.join(ROOT, "profiles", "experts_cfg1_traffic.json")
    if os.path.exists(prof_path):
        try:
            p = json.load(open(prof_path))
            traffic = float(p["dram_bytes_per_algorithmic_byte"]) * (up_bytes / prof_n)
        except Exception:
            traffic = None
    roofline = {"bound": "hbm", "achieved": up_gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": up_gbs / hbm_peak, "traffic": traffic,
                "kernel": "k_experts (gate_up + SwiGLU and down + scale, persistent)",
                "peak_source": f"{peak_src} hbm_gbs",
                "stage_ms_per_layer": {k_: v_ / prof_n for k_, v_ in stage_tot.items()}}

    # secondary: T=4 (MTP-verify width) on the same stack
    # secondary widths on the same stack: T=4 (MTP-verify width) and T=1
    # (batch-1 decode, config 0's width)
    def narrow(tokens):
        bufs_n = make_bufs(tokens)
        el_n = timed(tokens, bufs_n, args.steps, args.warmup)
        idx_n = bufs_n[2].cpu().numpy()
        u_n = [len(np.unique(idx_n[l])) for l in range(L)]
        b_n = sum(algorithmic_bytes(w, tokens, u) for u in u_n)
        st_n, kb_n, n_n = stage_profile(tokens, bufs_n, u_n)
        return {"tokens": tokens, "value": world * tokens * L * args.steps / el_n,
                "ms_per_step": el_n / args.steps * 1e3,
                "block_gbs": b_n * args.steps / el_n / 1e9 * (1 if world == 1 else world),
                "block_frac_hbm": b_n * args.steps / el_n / 1e9 / hbm_peak,
                "experts_gbs": kb_n / (st_n["experts"] / 1e3) / 1e9,
                "stage_ms_per_layer": {k_: v_ / n_n for k_, v_ in st_n.items()}}

    t4 = narrow(4) if T != 4 else None
    t1 = narrow(1) if T != 1 else None

    # end to end through the C ABI with HOST buffers (fw_moe_forward per layer)
    xh = torch.from_numpy(np.stack([synth.synth_input(input_seed(rank, l), T, H)
                                    for l in range(L)]).view(np.int16)).pin_memory()
    xh_np = xh.numpy().view(np.uint16)
    yh = torch.empty((L, T, H), dtype=torch.int16).pin_memory().numpy().view(np.uint16)
    ih = torch.empty((L, T, K), dtype=torch.int32).pin_memory().numpy()
    sh = torch.empty((L, T, K), dtype=torch.int16).pin_memory().numpy().view(np.uint16)
    lib = fw.library()

    def e2e_step():
        for l in range(L):
            rc = lib.fw_moe_forward(blk.handle, l, xh_np[l].ctypes.data, T, yh[l].ctypes.data,
                                    ih[l].ctypes.data, sh[l].ctypes.data)
            if rc != 0:
                raise fw.FwError(rc, lib.fw_last_error().decode())

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e2e_steps = max(1, args.steps // 2)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_el = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": world * T * L * e2e_steps / e2e_el, "unit": UNIT,
           "h2d_bytes_per_step": L * T * H * 2,
           "d2h_bytes_per_step": L * T * (H * 2 + K * 4 + K * 2),
           "api": "fw_moe_forward (synchronous, pinned host buffers), one call per layer"}

    blk.close()
    prefill = None if args.no_prefill else measure_prefill(args, rank, world, local_rank, peaks, stream,
                                                          max_over_ranks, barrier)
    ep = None
    if world > 1 and not args.no_ep:
        ep = measure_ep(args, rank, world, local_rank, peaks, stream, max_over_ranks, barrier, dist)
    cfg4 = None
    if not args.no_cfg4:
        cfg4 = measure_cfg4(args, rank, world, local_rank, peaks, stream, max_over_ranks, barrier, dist)

    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(w, os.cpu_count() or 1, budget_s=args.cpu_budget, rank=rank)
        # parity of this run's layer-0 outputs against the oracle (same inputs)
        import oracle as O
        shape = O.BlockShape(w["hidden"], w["intermediate"], w["shared_intermediate"],
                             w["experts"], K)
        Lw = O.SynthLayer(shape, layer_seed(0), 0.02, w["zipf"])
        x0 = synth.synth_input(input_seed(rank, 0), T, H)
        ry, ridx, rsc = O.block(shape, Lw, x0, threads=os.cpu_count() or 1)
        gy = bufs[1][0].cpu().numpy().view(np.uint16)
        gi = bufs[2][0].cpu().numpy()
        parity = {"layer": 0, "tokens": T, "indices_identical": bool(np.array_equal(gi, ridx)),
                  "bit_exact_tokens": int(np.all(gy == ry, axis=1).sum())}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded weights N(0,0.02)-like, inputs N(0,1) RMS-normalised)",
            "config": {"workload": w["name"], "layers": L, "tokens": T, "hidden": H,
                       "experts": w["experts"], "top_k": K, "intermediate": w["intermediate"],
                       "shared_intermediate": w["shared_intermediate"],
                       "parallelism": "replicas" if world > 1 else "single",
                       "l2": "no flush: every layer streams >126 MB of distinct weights",
                       "distinct_experts_per_layer_mean": float(np.mean(unique))},
            "stack_tokens_per_s": world * T * args.steps / el,
            "block_gbs": step_bytes * args.steps / el / 1e9 * world,
            "block_frac_hbm": step_bytes * args.steps / el / 1e9 / hbm_peak,
            "roofline": roofline,
            "gpu_launches": 4 * L * args.steps,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "parity_sample": parity,
            "t4": t4,
            "t1": t1,
            "prefill": prefill,
            "ep": ep,
            "cfg4": cfg4,
        }
        print(json.dumps(line), flush=True)


def measure_prefill(args, rank, world, local_rank, peaks, stream, max_over_ranks, barrier):
    """benchmark config 2 on the tensor-core prefill path: one block, T=8192
    tokens, Zipf-biased router.  CUDA events around `steps` forwards with
    device-resident inputs; a per-stage pass afterwards."""
    import torch

    import firewing_b200 as fw
    from firewing_b200 import synth

    p = PREFILL
    T, H, K = p["tokens"], p["hidden"], p["top_k"]
    cfg = fw.MoeConfig(H, p["intermediate"], p["shared_intermediate"], p["experts"], K,
                       max_tokens=T, layers=1)
    blk = fw.MoeBlock(cfg, device=local_rank)
    blk.synth_layer(0, p["seed"], 0.02, p["zipf"])
    x = torch.from_numpy(synth.synth_input(input_seed(rank, 0), T, H).view(np.int16)).cuda()
    y = torch.empty((T, H), dtype=torch.int16, device="cuda")
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((T, K), dtype=torch.int16, device="cuda")
    steps = max(3, args.steps // 5)
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            blk.forward_async(0, x, T, y, idx, sc, stream=stream)
    blk.sync(stream)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        blk.forward_async(0, x, T, y, idx, sc, stream=stream)
    e1.record(stream)
    e1.synchronize()
    blk.sync(stream)
    el = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    blk.profile(True)
    stages = {s_: 0.0 for s_ in fw.MoeBlock.STAGES}
    for _ in range(3):
        blk.forward_async(0, x, T, y, idx, sc, stream=stream)
        for k_, v_ in blk.profile_read().items():
            stages[k_] += v_ / 3
    blk.profile(False)
    ids = idx.cpu().numpy()
    counts = np.bincount(ids.ravel(), minlength=p["experts"])
    unique = int((counts > 0).sum())
    I, Is = p["intermediate"], p["shared_intermediate"]
    flops = 2 * 3 * H * I * T * K + 2 * 3 * H * Is * T
    wbytes = unique * 3 * H * I * 2 + 3 * H * Is * 2
    ex_s = stages["experts"] / 1e3
    tc_peak = float(peaks.get("bf16_tflops", 1590.0)) if peaks else 1590.0
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0)) if peaks else 6650.0
    blk.close()
    return {
        "workload": p["name"], "tokens": T, "layers": 1, "steps": steps,
        "value": world * T * steps / el, "unit": UNIT, "ms_per_step": el / steps * 1e3,
        "stage_ms": stages,
        "experts_tflops": flops / ex_s / 1e12,
        "experts_frac_tensor": flops / ex_s / 1e12 / tc_peak,
        "experts_weight_gbs": wbytes / ex_s / 1e9,
        "experts_frac_hbm": wbytes / ex_s / 1e9 / hbm_peak,
        "peak_source": "measured bf16_tflops / hbm_gbs" if peaks else "fallback",
        "hottest_expert_tokens": int(counts.max()), "distinct_experts": unique,
        "gpu_launches_per_step": 8,
        "kernels": "router logits (tcgen05), exact repair of the selectable logits (CUDA cores), route, "
                   "pair offsets, pair scatter, gate/up GEMM (tcgen05, SwiGLU epilogue), down GEMM "
                   "(tcgen05, weight epilogue), combine",
    }


def measure_cfg4(args, rank, world, local_rank, peaks, stream, max_over_ranks, barrier, dist):
    """benchmark config 4: 12 layers of the larger block at prefill width,
    8192 tokens per GPU per layer, Zipf-biased router.  One GPU at N = 1;
    expert parallelism over the N GPUs otherwise (rank r holds the experts
    e with e % N == r).  Whole-job token-layers/s and its per-GPU share,
    from which the expert-parallel efficiency against N = 1 follows."""
    import torch

    import firewing_b200 as fw
    from firewing_b200 import synth

    p = CFG4
    T, L = p["tokens"], p["layers"]
    H, K, E, I, Is = p["hidden"], p["top_k"], p["experts"], p["intermediate"], p["shared_intermediate"]
    blk = fw.MoeBlock(fw.MoeConfig(H, I, Is, E, K, max_tokens=T, layers=L), device=local_rank)
    if world > 1:
        uid = [fw.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        blk.ep_init(rank, world, uid[0])
    for l in range(L):
        blk.synth_layer(l, 100 + l, 0.02, p["zipf"])
    x = torch.from_numpy(np.stack([synth.synth_input(input_seed(rank, l), T, H) for l in range(L)])
                         .view(np.int16)).cuda()
    y = torch.empty((L, T, H), dtype=torch.int16, device="cuda")
    idx = torch.empty((L, T, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((L, T, K), dtype=torch.int16, device="cuda")

    def step():
        for l in range(L):
            blk.forward_async(l, x[l], T, y[l], idx[l], sc[l], stream=stream)

    steps = 3
    for _ in range(2):
        step()
    blk.sync(stream)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    e1.synchronize()
    blk.sync(stream)
    el = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    blk.close()
    flops = 2 * 3 * H * I * T * K + 2 * 3 * H * Is * T  # per GPU per layer
    tc_peak = float(peaks.get("bf16_tflops", 1590.0)) if peaks else 1590.0
    value = world * T * L * steps / el
    return {
        "workload": p["name"], "n_gpus": world, "tokens_per_gpu": T, "layers": L, "steps": steps,
        "value": value, "per_gpu_value": value / world, "unit": UNIT, "ms_per_layer": el / steps / L * 1e3,
        "expert_tflops_per_gpu": flops * L * steps / el / 1e12,
        "expert_frac_tensor_per_gpu": flops * L * steps / el / 1e12 / tc_peak,
        "parallelism": f"ep{world}" if world > 1 else "single",
        "note": "expert-parallel efficiency = per_gpu_value at N / value at N = 1",
    }


def measure_ep(args, rank, world, local_rank, peaks, stream, max_over_ranks, barrier, dist):
    """benchmark config 3 on `world` GPUs with expert parallelism: decode of
    256 tokens per layer in total (256/world per rank), uniform routing, a
    48-layer stack at 8 GPUs (64 experts per GPU), 24 layers at 2 or 4.
    Rank r holds the experts e with e % world == r of every layer; each
    forward gathers every rank's tokens, runs the local experts, returns the
    weighted rows to their owners over NCCL and sums them there."""
    import torch

    import firewing_b200 as fw
    from firewing_b200 import synth

    p = EP
    T_l = p["tokens"] // world
    L = p["layers_8"] if world >= 8 else p["layers"]
    H, K, E, I, Is = p["hidden"], p["top_k"], p["experts"], p["intermediate"], p["shared_intermediate"]
    uid = [fw.ep_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    blk = fw.MoeBlock(fw.MoeConfig(H, I, Is, E, K, max_tokens=T_l, layers=L), device=local_rank)
    blk.ep_init(rank, world, uid[0])
    for l in range(L):
        blk.synth_layer(l, layer_seed(l), 0.02, False)
    xs = np.stack([synth.synth_input(input_seed(rank, l), T_l, H) for l in range(L)])
    x = torch.from_numpy(xs.view(np.int16)).cuda()
    y = torch.empty((L, T_l, H), dtype=torch.int16, device="cuda")
    idx = torch.empty((L, T_l, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((L, T_l, K), dtype=torch.int16, device="cuda")

    def step():
        for l in range(L):
            blk.forward_async(l, x[l], T_l, y[l], idx[l], sc[l], stream=stream)

    steps = max(3, args.steps // 2)
    for _ in range(max(3, args.warmup)):
        step()
    blk.sync(stream)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    e1.synchronize()
    blk.sync(stream)
    el = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    # this rank's distinct local experts per layer (from every rank's picks)
    ids = idx.cpu().numpy()
    t_ids = torch.from_numpy(ids.astype(np.int32)).cuda()
    all_ids = [torch.empty_like(t_ids) for _ in range(world)]
    dist.all_gather(all_ids, t_ids)
    cat = np.concatenate([a.cpu().numpy() for a in all_ids], axis=1)
    local_u = [int((np.unique(cat[l]) % world == rank).sum()) for l in range(L)]
    layer_bytes = [u * 3 * H * I * 2 + E * H * 2 + 3 * H * Is * 2 for u in local_u]
    gbs = sum(layer_bytes) * steps / el / 1e9
    gbs = max_over_ranks(-gbs) * -1  # slowest rank's streaming rate
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0)) if peaks else 6650.0
    blk.close()
    return {
        "workload": p["name"].format(world=world, per=E // world, layers=L),
        "tokens_per_layer": T_l * world, "tokens_per_rank": T_l, "layers": L, "steps": steps,
        "value": T_l * world * L * steps / el, "unit": UNIT, "ms_per_step": el / steps * 1e3,
        "per_gpu_gbs_min": gbs, "per_gpu_frac_hbm_min": gbs / hbm_peak,
        "parallelism": f"ep{world} (experts {E // world} per GPU) + dp tokens",
        "exchange": "NCCL all-gather (rows, ids, weights) + grouped send/recv of weighted rows",
    }


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="cfg1", choices=sorted(WORKLOADS))
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--tokens", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-2 prefill line item")
    ap.add_argument("--no-ep", action="store_true", help="skip the config-3 expert-parallel line item (N > 1)")
    ap.add_argument("--no-cfg4", action="store_true", help="skip the config-4 prefill line item")
    ap.add_argument("--only-prefill", action="store_true",
                    help="run only the config-2 prefill measurement and print it (for ncu captures)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--minimal", action="store_true",
                    help="timed steps only (no T=4 pass, e2e, stage profile or CPU leg); "
                         "for ncu captures")
    args = ap.parse_args()
    w = dict(WORKLOADS[args.workload])
    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference(args, w, rank)
        return
    if args.only_prefill:
        import torch

        torch.cuda.set_device(local_rank)
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except Exception:
            pass
        pre = measure_prefill(args, rank, 1, local_rank, peaks, torch.cuda.Stream(), lambda v: v, lambda: None)
        print(json.dumps({"only_prefill": True, "prefill": pre}), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, w, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
