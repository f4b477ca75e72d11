"""CPU model of the prefill router (k_router_tc + k_router_fix): approximate
logits summed in another order, the interval test, the exact repair.

It checks the two claims the kernels rest on against the oracle's exact
logits (the reference's 32-partial schedule, src/expert.rs:514-552):
  - every reference logit lies in its interval [f(a - delta), f(a + delta)],
    delta = 2^-10 * |w_e|_2 * |x_t|_2, f = bf16 rounding plus the bias;
  - routing the repaired logits (exact for every candidate, the rounded
    approximation elsewhere) selects exactly the reference's experts, with
    scores within one bf16 step.
A float32 matrix product (BLAS, its own order of f32 additions) stands in
for the tensor core's accumulation.
"""
import numpy as np
import pytest

import oracle as O

H, E, K = 2048, 512, 10


def total_key(bits: np.ndarray) -> np.ndarray:
    b = bits.astype(np.uint32)
    return np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)


def biased(v: np.ndarray, bias) -> np.ndarray:
    b = O.f32_to_bf16(v.astype(np.float32))
    if bias is not None:
        b = O.f32_to_bf16((O.bf16_to_f32(b) + bias).astype(np.float32))
    return b


def norm_bound(rows: np.ndarray) -> np.ndarray:
    ss = np.sum(rows.astype(np.float32) ** 2, axis=-1, dtype=np.float32)
    up = np.nextafter(np.sqrt(ss * np.float32(1.00390625)), np.float32(np.inf))
    return np.maximum(up, np.float32(2.0 ** -60)).astype(np.float32)


@pytest.mark.parametrize("zipf,seed", [(False, 3), (True, 4)])
def test_repair_selects_reference_experts(zipf, seed):
    shape = O.BlockShape(hidden=H, intermediate=512, shared_intermediate=512, experts=E, top_k=K)
    layer = O.SynthLayer(shape, seed, 0.02, zipf)
    x = O.synth_input(seed + 100, 96, H)
    ridx, rsc, rlog = O.router(shape, layer, x)
    W = O.bf16_to_f32(layer.router).reshape(E, H)
    X = O.bf16_to_f32(x)
    approx = (X @ W.T).astype(np.float32)
    d = np.nextafter((np.float32(2.0 ** -10) * norm_bound(X)[:, None] * norm_bound(W)[None, :]).astype(np.float32),
                     np.float32(np.inf))
    lo = total_key(biased(np.nextafter((approx - d).astype(np.float32), np.float32(-np.inf)), layer.bias))
    hi = total_key(biased(np.nextafter((approx + d).astype(np.float32), np.float32(np.inf)), layer.bias))
    ref = total_key(rlog)
    assert np.all(lo <= ref) and np.all(ref <= hi), "reference logit outside its interval"
    tau = -np.sort(-lo, axis=1)[:, K - 1]
    cand = hi >= tau[:, None]
    repaired = np.where(cand, rlog, biased(approx, layer.bias)).astype(np.uint16)
    for t in range(x.shape[0]):
        assert set(ridx[t].tolist()) <= set(np.nonzero(cand[t])[0].tolist())
        idx, sc = O.route(np.ascontiguousarray(repaired[t]), K)
        assert np.array_equal(idx, ridx[t]), t
        assert int(np.abs(sc.astype(np.int32) - rsc[t].astype(np.int32)).max()) <= 1, t
    assert cand.sum(axis=1).mean() < 20, "the exact repair stays a handful of dots per token"


def test_interval_without_repair_would_not_suffice():
    """The rounded approximations alone differ from the reference's logits
    somewhere (that is why the repair exists)."""
    shape = O.BlockShape(hidden=H, intermediate=512, shared_intermediate=512, experts=E, top_k=K)
    layer = O.SynthLayer(shape, 5, 0.02, False)
    x = O.synth_input(105, 96, H)
    _, _, rlog = O.router(shape, layer, x)
    approx = (O.bf16_to_f32(x) @ O.bf16_to_f32(layer.router).reshape(E, H).T).astype(np.float32)
    assert np.any(biased(approx, None) != rlog)
