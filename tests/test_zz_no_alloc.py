"""fw_moe_forward_noalloc against the handle-based block forward.

The no-allocation entry point serves callers that cannot cudaMalloc (a
framework whose caching allocator already holds the device's memory, or a
latency-critical loop that must not synchronise the device through
cudaMalloc/cudaFree).  It runs the same block over caller-owned device
buffers with its scratch in a static 8 MiB device array.  Two calls in a row
(different inputs and token counts, so stale scratch would show) must match
the existing entry point within the parity tolerance of the other tests --
in practice bit for bit, since both run the same kernels.

This file sorts last so a run that stops at the first failure has already
run every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402

MAX_ABS = 2e-2
REL_L2 = 1e-3

SHAPES = [
    dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4),
    dict(hidden=1024, intermediate=256, shared_intermediate=256, experts=128, top_k=8),
]


def dev(a: np.ndarray):
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()


def device_weights(shape: dict, seed: int, zipf: bool) -> dict:
    layer = O.SynthLayer(O.BlockShape(**shape), seed, 0.02, zipf)
    for e in range(shape["experts"]):
        layer.expert(e)
    w = {
        "router": dev(layer.router),
        "gate_up": dev(np.concatenate([layer.gate_up[e] for e in range(shape["experts"])])),
        "down": dev(np.concatenate([layer.down[e] for e in range(shape["experts"])])),
        "shared_gate": dev(layer.shared_gate),
        "shared_up": dev(layer.shared_up),
        "shared_down": dev(layer.shared_down),
        "shared_gate_w": dev(layer.shared_gate_w),
    }
    if zipf:
        w["logit_bias"] = dev(layer.bias)
    return w


def close(y: np.ndarray, r: np.ndarray) -> bool:
    yf = O.bf16_to_f32(y).astype(np.float64)
    rf = O.bf16_to_f32(r).astype(np.float64)
    max_abs = float(np.abs(yf - rf).max())
    rel = float(np.linalg.norm(yf - rf) / max(np.linalg.norm(rf), 1e-30))
    return max_abs <= MAX_ABS and rel <= REL_L2


# Token counts of the two calls.  At T <= 4 the handle path takes other
# kernels than at wider T (for hidden a multiple of 256: the partial-major
# router at T = 1, the small-width expert kernel on its re-laid-out banks),
# while this entry point always runs the generic router and expert kernel on
# reference-layout weights; both must still agree bit for bit.
@pytest.mark.parametrize("shape_i,zipf,tokens", [(0, False, (32, 7)), (1, False, (32, 7)), (1, True, (32, 7)),
                                                 (1, False, (1, 3)), (1, True, (3, 1))])
def test_noalloc_matches_handle_forward_twice(shape_i, zipf, tokens):
    shape = SHAPES[shape_i]
    H, K = shape["hidden"], shape["top_k"]
    cfg = fw.MoeConfig(**shape, max_tokens=32, layers=1)
    w = device_weights(shape, 40 + shape_i, zipf)
    blk = fw.MoeBlock(cfg)
    blk.load_layer(0, w["router"], w["gate_up"], w["down"], w["shared_gate"], w["shared_up"],
                   w["shared_down"], w["shared_gate_w"], w.get("logit_bias"))
    stream = torch.cuda.current_stream()
    for call, T in enumerate(tokens):
        x = dev(O.synth_input(500 + call, T, H))
        y_ref = torch.empty((T, H), dtype=torch.int16, device="cuda")
        i_ref = torch.empty((T, K), dtype=torch.int32, device="cuda")
        s_ref = torch.empty((T, K), dtype=torch.int16, device="cuda")
        blk.forward_async(0, x, T, y_ref, i_ref, s_ref, stream=stream)
        blk.sync(stream)
        y = torch.full((T, H), -1, dtype=torch.int16, device="cuda")
        idx = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
        sc = torch.full((T, K), -1, dtype=torch.int16, device="cuda")
        fw.forward_noalloc(cfg, w, x, T, y, idx, sc, stream=stream)
        torch.cuda.synchronize()
        assert np.array_equal(idx.cpu().numpy(), i_ref.cpu().numpy()), f"call {call}"
        assert np.array_equal(sc.cpu().numpy(), s_ref.cpu().numpy()), f"call {call}"
        yn = y.cpu().numpy().view(np.uint16)
        yr = y_ref.cpu().numpy().view(np.uint16)
        assert close(yn, yr), f"call {call}"
        assert np.array_equal(yn, yr), f"call {call}"
    blk.close()


def test_noalloc_topk_buffers_optional():
    shape = SHAPES[0]
    cfg = fw.MoeConfig(**shape, max_tokens=8, layers=1)
    w = device_weights(shape, 3, False)
    T, H = 8, shape["hidden"]
    x = dev(O.synth_input(9, T, H))
    y1 = torch.empty((T, H), dtype=torch.int16, device="cuda")
    y2 = torch.empty((T, H), dtype=torch.int16, device="cuda")
    idx = torch.empty((T, shape["top_k"]), dtype=torch.int32, device="cuda")
    sc = torch.empty((T, shape["top_k"]), dtype=torch.int16, device="cuda")
    fw.forward_noalloc(cfg, w, x, T, y1, idx, sc)
    fw.forward_noalloc(cfg, w, x, T, y2)
    assert torch.equal(y1, y2)


def test_noalloc_rejects_scratch_beyond_the_static_area():
    shape = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10)
    cfg = fw.MoeConfig(**shape, max_tokens=256, layers=1)
    dummy = torch.zeros(64, dtype=torch.int16, device="cuda")
    w = {k: dummy for k in ("router", "gate_up", "down", "shared_gate", "shared_up",
                            "shared_down", "shared_gate_w")}
    with pytest.raises(fw.FwError) as e:
        fw.forward_noalloc(cfg, w, dummy, 256, dummy)
    assert e.value.code == fw.FW_EINVAL
    assert "scratch" in e.value.message


def test_noalloc_scratch_limit_at_config0():
    # Config 0 (H=2048, I=Is=512, E=512, K=10): T=121 fits the 8 MiB area,
    # T=122 does not.  Zero weights are enough to run the forward.
    shape = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10)
    H, I, E = shape["hidden"], shape["intermediate"], shape["experts"]
    cfg = fw.MoeConfig(**shape, max_tokens=122, layers=1)
    z = lambda n: torch.zeros(n, dtype=torch.int16, device="cuda")  # noqa: E731
    w = {"router": z(E * H), "gate_up": z(E * 2 * I * H), "down": z(E * H * I), "shared_gate": z(I * H),
         "shared_up": z(I * H), "shared_down": z(H * I), "shared_gate_w": z(H)}
    x = dev(O.synth_input(77, 122, H))
    y = torch.empty((122, H), dtype=torch.int16, device="cuda")
    idx = torch.empty((122, shape["top_k"]), dtype=torch.int32, device="cuda")
    fw.forward_noalloc(cfg, w, x, 121, y, idx)
    torch.cuda.synchronize()
    # all logits equal: the tie rule selects experts 0..K-1 in index order
    assert np.array_equal(idx[:121].cpu().numpy(), np.tile(np.arange(10, dtype=np.int32), (121, 1)))
    with pytest.raises(fw.FwError) as e:
        fw.forward_noalloc(cfg, w, x, 122, y, idx)
    assert e.value.code == fw.FW_EINVAL
    assert "scratch" in e.value.message
    del w
    torch.cuda.empty_cache()


def test_noalloc_reports_nan_logits():
    shape = SHAPES[0]
    cfg = fw.MoeConfig(**shape, max_tokens=4, layers=1)
    w = device_weights(shape, 5, False)
    xh = O.synth_input(6, 4, shape["hidden"])
    xh[1, 3] = 0x7FC0
    y = torch.empty((4, shape["hidden"]), dtype=torch.int16, device="cuda")
    with pytest.raises(fw.FwError) as e:
        fw.forward_noalloc(cfg, w, dev(xh), 4, y)
    assert e.value.code == fw.FW_ENAN
