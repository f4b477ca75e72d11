"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bar (the target's stated tolerance): selected expert indices identical except where
router logits tie; block output within max-abs 2e-2 and relative-L2 1e-3.
The CUDA path keeps the reference's reduction order, so outputs are expected
bit-identical; the only licensed difference is a renormalised score one bf16
ulp apart, from the router softmax's exp (correctly rounded on the GPU,
host-libm expf in the oracle).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import firewing_b200 as fw  # noqa: E402

MAX_ABS = 2e-2
REL_L2 = 1e-3


def dev(a: np.ndarray):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    return torch.from_numpy(a).cuda()


def host(t, dtype=np.uint16):
    return t.cpu().numpy().view(dtype)


def rand_bf16(rng, shape, scale=1.0):
    return O.f32_to_bf16((rng.standard_normal(size=shape) * scale).astype(np.float32))


def ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.abs(a.astype(np.int32) - b.astype(np.int32))


def assert_block_close(y, y_ref, idx, idx_ref, sc, sc_ref, logits_ref):
    T, K = idx.shape
    for t in range(T):
        assert O.equivalent_topk_order(idx_ref[t], idx[t], logits_ref[t]), f"token {t}"
    assert np.array_equal(idx, idx_ref), "same logits + same tie rule => identical selection"
    assert int(ulp_diff(sc, sc_ref).max()) <= 1
    yf, rf = O.bf16_to_f32(y).astype(np.float64), O.bf16_to_f32(y_ref).astype(np.float64)
    assert np.all(np.isfinite(yf))
    max_abs = float(np.abs(yf - rf).max())
    rel = float(np.linalg.norm(yf - rf) / max(np.linalg.norm(rf), 1e-30))
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)
    exact_tokens = np.all(sc == sc_ref, axis=1)
    assert np.array_equal(y[exact_tokens], y_ref[exact_tokens]), "bit-exact when scores match"


# ---------------------------------------------------------------------------
# primitives

@pytest.mark.parametrize("rows,cols,T", [(1, 32, 1), (17, 96, 3), (513, 2048, 8), (100, 512, 9),
                                         (64, 3072, 5), (40, 64, 17)])
def test_linear_bit_exact(rows, cols, T):
    rng = np.random.default_rng(rows * 1000 + cols + T)
    w = rand_bf16(rng, (rows, cols), 0.02)
    x = rand_bf16(rng, (T, cols))
    y = torch.empty((T, rows), dtype=torch.int16, device="cuda")
    fw.linear_bf16(dev(w), dev(x), rows, cols, T, y)
    torch.cuda.synchronize()
    got = host(y)
    for t in range(T):
        assert np.array_equal(got[t], O.linear_bf16(w.ravel(), x[t].copy(), rows, cols)), t


def test_linear_rejects_bad_shapes():
    z = torch.zeros(64, dtype=torch.int16, device="cuda")
    with pytest.raises(fw.FwError):
        fw.linear_bf16(z, z, 1, 33, 1, z)


def test_swiglu_exhaustive_over_gate_bits():
    gates = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    finite = (gates & 0x7F80) != 0x7F80
    gates = gates[finite].copy()
    rng = np.random.default_rng(5)
    ups = rand_bf16(rng, gates.shape)
    out = torch.empty(gates.size, dtype=torch.int16, device="cuda")
    fw.swiglu_bf16(dev(gates), dev(ups), gates.size, out)
    torch.cuda.synchronize()
    assert np.array_equal(host(out), O.swiglu_bf16(gates, ups))


@pytest.mark.parametrize("E,K,T,scale", [(512, 10, 40, 1.0), (512, 10, 33, 0.05), (64, 4, 9, 1.0),
                                         (1024, 32, 5, 1.0), (32, 1, 3, 1.0)])
def test_route_matches_oracle(E, K, T, scale):
    rng = np.random.default_rng(E + K + T)
    logits = rand_bf16(rng, (T, E), scale)
    idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
    sc = torch.empty((T, K), dtype=torch.int16, device="cuda")
    fw.route_bf16(dev(logits), T, E, K, idx, sc)
    gi, gs = idx.cpu().numpy(), host(sc)
    for t in range(T):
        ri, rs = O.route(logits[t].copy(), K)
        assert np.array_equal(gi[t], ri)
        assert int(ulp_diff(gs[t], rs).max()) <= 1


def test_route_tie_known_answers():
    # src/decoder_layer.rs:666-679 under the deterministic tie rule
    z = np.zeros((2, 512), dtype=np.uint16)
    for i in (10, 20, 30, 40, 50, 60, 70, 80, 90):
        z[1, i] = O.to_bf16(1.0)
    idx = torch.empty((2, 10), dtype=torch.int32, device="cuda")
    sc = torch.empty((2, 10), dtype=torch.int16, device="cuda")
    fw.route_bf16(dev(z), 2, 512, 10, idx, sc)
    gi = idx.cpu().numpy()
    assert gi[0].tolist() == list(range(10))
    assert gi[1].tolist() == [10, 20, 30, 40, 50, 60, 70, 80, 90, 0]


def test_route_rejects_nan():
    z = np.zeros((3, 64), dtype=np.uint16)
    z[1, 5] = 0x7FC1
    idx = torch.empty((3, 4), dtype=torch.int32, device="cuda")
    sc = torch.empty((3, 4), dtype=torch.int16, device="cuda")
    with pytest.raises(fw.FwError) as e:
        fw.route_bf16(dev(z), 3, 64, 4, idx, sc)
    assert e.value.code == fw.FW_ENAN
    fw.route_bf16(dev(np.zeros((3, 64), dtype=np.uint16)), 3, 64, 4, idx, sc)  # recovers


def test_topk_dropin_matches_oracle():
    rng = np.random.default_rng(9)
    for trial in range(5):
        v = rand_bf16(rng, (512,))
        for k in (1, 10, 32):
            assert fw.topk_bf16(v, k) == O.topk_bf16(v, k).tolist()


# ---------------------------------------------------------------------------
# whole block

SMALL = dict(hidden=256, intermediate=128, shared_intermediate=192, experts=64, top_k=4)
CFG0 = dict(hidden=2048, intermediate=512, shared_intermediate=512, experts=512, top_k=10)


def run_pair(shape: dict, seed: int, T: int, zipf: bool = False, x=None, max_tokens=None):
    cfg = fw.MoeConfig(**shape, max_tokens=max_tokens or max(T, 1), layers=1)
    blk = fw.MoeBlock(cfg)
    # this file checks the bit-exact decode path: pinned up to its 256-token
    # limit (shapes with a prefill path take it from 96 tokens by default)
    blk.set_prefill_min_tokens(1 << 20)
    blk.synth_layer(0, seed, 0.02, zipf)
    bshape = O.BlockShape(**shape)
    layer = O.SynthLayer(bshape, seed, 0.02, zipf)
    if x is None:
        x = O.synth_input(seed + 1000, T, shape["hidden"])
    y, idx, sc = blk.forward(0, x)
    ry, ridx, rsc, taps = O.block(bshape, layer, x, threads=8, taps=True)
    return blk, layer, x, (y, idx, sc), (ry, ridx, rsc, taps)


@pytest.mark.parametrize("T", [1, 3, 17, 64])
def test_block_small_shape(T):
    _, _, _, got, ref = run_pair(SMALL, 3, T)
    assert_block_close(got[0], ref[0], got[1], ref[1], got[2], ref[2], ref[3]["logits"])


def test_block_small_shape_max_tokens_256_zipf():
    _, _, _, got, ref = run_pair(SMALL, 4, 256, zipf=True)
    assert_block_close(got[0], ref[0], got[1], ref[1], got[2], ref[2], ref[3]["logits"])


# T <= 4 runs the small-width expert kernel (T = 2: two-token passes; T = 3:
# four-wide passes with a padded token); 64 the eight-warp kernel.
@pytest.mark.parametrize("T,zipf", [(1, False), (2, False), (3, True), (4, False), (64, False), (64, True)])
def test_block_config0_shape(T, zipf):
    _, _, _, got, ref = run_pair(CFG0, 0, T, zipf=zipf)
    assert_block_close(got[0], ref[0], got[1], ref[1], got[2], ref[2], ref[3]["logits"])


CFG4 = dict(hidden=3072, intermediate=768, shared_intermediate=768, experts=512, top_k=10)


@pytest.mark.parametrize("T", [1, 4, 33])
def test_block_config4_shape_zipf(T):
    # Benchmark config 4's block (H=3072, I=Is=768) on the decode path.
    _, _, _, got, ref = run_pair(CFG4, 3, T, zipf=True)
    assert_block_close(got[0], ref[0], got[1], ref[1], got[2], ref[2], ref[3]["logits"])


# A hidden size that is not a multiple of 256: the decode router without the
# partial-major copy (and no prefill path).
ODD_H = dict(hidden=192, intermediate=128, shared_intermediate=128, experts=64, top_k=4)


@pytest.mark.parametrize("T", [1, 6])
def test_block_hidden_not_multiple_of_256(T):
    _, _, _, got, ref = run_pair(ODD_H, 6, T, zipf=True)
    assert_block_close(got[0], ref[0], got[1], ref[1], got[2], ref[2], ref[3]["logits"])


def test_block_all_ties_input():
    # x = 0 -> every logit 0: selection 0..K-1, equal scores (tie rule).
    x = np.zeros((2, SMALL["hidden"]), dtype=np.uint16)
    _, _, _, got, ref = run_pair(SMALL, 5, 2, x=x)
    assert got[1][0].tolist() == list(range(SMALL["top_k"]))
    assert_block_close(got[0], ref[0], got[1], ref[1], got[2], ref[2], ref[3]["logits"])


def test_block_host_weights_equal_device_synth():
    shape = SMALL
    cfg = fw.MoeConfig(**shape, max_tokens=8, layers=2)
    blk = fw.MoeBlock(cfg)
    blk.synth_layer(0, 21)
    L = O.SynthLayer(O.BlockShape(**shape), 21)
    for e in range(shape["experts"]):
        L.expert(e)
    gate_up = np.concatenate([L.gate_up[e] for e in range(shape["experts"])])
    down = np.concatenate([L.down[e] for e in range(shape["experts"])])
    blk.load_layer(1, L.router, gate_up, down, L.shared_gate, L.shared_up, L.shared_down,
                   L.shared_gate_w)
    x = O.synth_input(77, 8, shape["hidden"])
    a = blk.forward(0, x)
    b = blk.forward(1, x)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)


def test_block_async_device_buffers_match_sync():
    shape = SMALL
    cfg = fw.MoeConfig(**shape, max_tokens=16, layers=1)
    blk = fw.MoeBlock(cfg)
    blk.synth_layer(0, 8)
    x = O.synth_input(9, 16, shape["hidden"])
    y_ref, i_ref, s_ref = blk.forward(0, x)
    xd = dev(x)
    y = torch.empty((16, shape["hidden"]), dtype=torch.int16, device="cuda")
    idx = torch.empty((16, shape["top_k"]), dtype=torch.int32, device="cuda")
    sc = torch.empty((16, shape["top_k"]), dtype=torch.int16, device="cuda")
    stream = torch.cuda.current_stream()
    blk.forward_async(0, xd, 16, y, idx, sc, stream=stream)
    blk.sync(stream)
    assert np.array_equal(host(y), y_ref)
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    assert np.array_equal(host(sc), s_ref)


def test_block_errors_fail_closed_and_recover():
    shape = SMALL
    cfg = fw.MoeConfig(**shape, max_tokens=4, layers=2)
    blk = fw.MoeBlock(cfg)
    blk.synth_layer(0, 1)
    x = O.synth_input(2, 4, shape["hidden"])
    with pytest.raises(fw.FwError) as e:
        blk.forward(1, x)  # layer 1 never loaded
    assert e.value.code == fw.FW_EINVAL
    with pytest.raises(fw.FwError) as e:
        blk.forward(0, np.zeros((5, shape["hidden"]), dtype=np.uint16))  # > max_tokens
    assert e.value.code == fw.FW_EINVAL
    bad = x.copy()
    bad[2, 7] = 0x7FC0  # NaN input -> NaN router logits
    with pytest.raises(fw.FwError) as e:
        blk.forward(0, bad)
    assert e.value.code == fw.FW_ENAN
    y, idx, sc = blk.forward(0, x)  # the handle stays usable
    ry, ridx, rsc = O.block(O.BlockShape(**shape), O.SynthLayer(O.BlockShape(**shape), 1), x)
    assert np.array_equal(idx, ridx)
    empty = blk.forward(0, np.zeros((0, shape["hidden"]), dtype=np.uint16))
    assert empty[0].shape == (0, shape["hidden"])
