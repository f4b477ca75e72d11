"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle is a plain-C restatement of the reference crate's CPU arithmetic
for the sparse-MoE block (see fw_oracle.c for the file:line citations).  Only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module, and only as the checker / the timed CPU reference: the product
package ``firewing_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libfw_oracle.so")
_SHIM_PATH = os.path.join(_HERE, "_ref", "libtopk_shim.so")

u16p = ctypes.POINTER(ctypes.c_uint16)
i32p = ctypes.POINTER(ctypes.c_int32)
f32p = ctypes.POINTER(ctypes.c_float)


class Shape(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("shared_intermediate", ctypes.c_int32),
        ("experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
    ]


class _Layer(ctypes.Structure):
    _fields_ = [
        ("router", u16p),
        ("gate_up", ctypes.POINTER(u16p)),
        ("down", ctypes.POINTER(u16p)),
        ("shared_gate", u16p),
        ("shared_up", u16p),
        ("shared_down", u16p),
        ("shared_gate_w", u16p),
        ("logit_bias", f32p),
    ]


class _Taps(ctypes.Structure):
    _fields_ = [("logits", u16p), ("routed", u16p), ("gated_shared", u16p)]


class InputSpec(ctypes.Structure):
    _fields_ = [
        ("multiplier", ctypes.c_int64),
        ("add", ctypes.c_int64),
        ("modulus", ctypes.c_int64),
        ("center", ctypes.c_int64),
        ("divisor", ctypes.c_int64),
        ("sparse_stride", ctypes.c_uint64),
    ]


def build(reference: Optional[str] = None) -> None:
    """Compile the oracle with oracle/Makefile, and the reference's top-k
    shim from its source when the firewing source tree is given (argument,
    or the FIREWING_REFERENCE environment variable)."""
    subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)
    ref = reference or os.environ.get("FIREWING_REFERENCE")
    if ref and os.path.isfile(os.path.join(ref, "native", "topk_shim.cpp")):
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={os.path.abspath(ref)}"], check=True)


_lib = None


class _HcLayer(ctypes.Structure):
    _fields_ = [("norm", u16p), ("mix_down", u16p), ("mix_up", u16p), ("inject", u16p)]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.fwo_to_bf16.restype = ctypes.c_uint16
        L.fwo_to_bf16.argtypes = [ctypes.c_float]
        L.fwo_from_bf16.restype = ctypes.c_float
        L.fwo_from_bf16.argtypes = [ctypes.c_uint16]
        for name in ("fwo_dot_bf16", "fwo_dot_forward"):
            getattr(L, name).restype = ctypes.c_float
            getattr(L, name).argtypes = [u16p, u16p, ctypes.c_size_t]
        L.fwo_linear_bf16.argtypes = [u16p, u16p, ctypes.c_size_t, ctypes.c_size_t, u16p]
        L.fwo_swiglu_bf16.argtypes = [u16p, u16p, ctypes.c_size_t, u16p]
        L.fwo_sigmoid_bf16.restype = ctypes.c_uint16
        L.fwo_sigmoid_bf16.argtypes = [ctypes.c_uint16]
        L.fwo_add_bf16.restype = ctypes.c_uint16
        L.fwo_add_bf16.argtypes = [ctypes.c_uint16, ctypes.c_uint16]
        L.fwo_build_silu_lut.argtypes = [u16p]
        L.fwo_build_sigmoid_lut.argtypes = [u16p]
        L.fwo_topk_bf16.argtypes = [u16p, ctypes.c_size_t, ctypes.c_size_t, i32p]
        L.fwo_route.argtypes = [u16p, ctypes.c_size_t, ctypes.c_size_t, i32p, u16p]
        L.fwo_equivalent_topk_order.argtypes = [i32p, i32p, ctypes.c_size_t, u16p]
        L.fwo_router.argtypes = [ctypes.POINTER(Shape), ctypes.POINTER(_Layer), u16p,
                                 ctypes.c_int32, i32p, u16p, u16p]
        L.fwo_block.argtypes = [ctypes.POINTER(Shape), ctypes.POINTER(_Layer), u16p,
                                ctypes.c_int32, u16p, i32p, u16p, ctypes.POINTER(_Taps),
                                ctypes.c_int32]
        L.fwo_splitmix64_key.restype = ctypes.c_uint64
        L.fwo_splitmix64_key.argtypes = [ctypes.c_uint64, ctypes.c_uint32]
        L.fwo_synth_scale.restype = ctypes.c_float
        L.fwo_synth_scale.argtypes = [ctypes.c_float]
        L.fwo_synth_bf16.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64,
                                     ctypes.c_size_t, ctypes.c_float, u16p]
        L.fwo_synth_input.argtypes = [ctypes.c_uint64, ctypes.c_int32, ctypes.c_int32, u16p]
        L.fwo_zipf_bias.argtypes = [ctypes.c_int32, f32p]
        L.fwo_make_hidden.argtypes = [ctypes.c_size_t, ctypes.POINTER(InputSpec), u16p]
        L.fwo_inner_square_sum.restype = ctypes.c_float
        L.fwo_inner_square_sum.argtypes = [f32p, ctypes.c_size_t]
        L.fwo_grouped_rms.argtypes = [u16p, u16p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float, u16p]
        L.fwo_four_stream_mean.restype = ctypes.c_float
        L.fwo_four_stream_mean.argtypes = [f32p]
        L.fwo_hc_pre.argtypes = [u16p, ctypes.POINTER(_HcLayer), ctypes.c_size_t, ctypes.c_size_t, u16p, u16p,
                                 u16p]
        L.fwo_hc_post.argtypes = [u16p, u16p, u16p, ctypes.c_size_t, u16p]
        _lib = L
    return _lib


def _p16(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(u16p)


def _p32(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(i32p)


def _pf(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(f32p)


# ---- scalar / vector primitives -------------------------------------------

def to_bf16(x: float) -> int:
    return int(lib().fwo_to_bf16(ctypes.c_float(x)))


def from_bf16(b: int) -> float:
    return float(lib().fwo_from_bf16(b))


def bf16_array(values: Sequence[float]) -> np.ndarray:
    return np.array([to_bf16(v) for v in values], dtype=np.uint16)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Vectorised copy of the reference's RNE formula (src/expert.rs:315-318)."""
    bits = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def dot_bf16(a: np.ndarray, b: np.ndarray) -> float:
    return float(lib().fwo_dot_bf16(_p16(a), _p16(b), a.size))


def dot_forward(a: np.ndarray, b: np.ndarray) -> float:
    return float(lib().fwo_dot_forward(_p16(a), _p16(b), a.size))


def linear_bf16(w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty(rows, dtype=np.uint16)
    lib().fwo_linear_bf16(_p16(w), _p16(x), rows, cols, _p16(out))
    return out


def swiglu_bf16(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    out = np.empty(gate.size, dtype=np.uint16)
    lib().fwo_swiglu_bf16(_p16(gate), _p16(up), gate.size, _p16(out))
    return out


def sigmoid_bf16(v: int) -> int:
    return int(lib().fwo_sigmoid_bf16(v))


def add_bf16(a: int, b: int) -> int:
    return int(lib().fwo_add_bf16(a, b))


def silu_lut() -> np.ndarray:
    out = np.empty(65536, dtype=np.uint16)
    lib().fwo_build_silu_lut(_p16(out))
    return out


def sigmoid_lut() -> np.ndarray:
    out = np.empty(65536, dtype=np.uint16)
    lib().fwo_build_sigmoid_lut(_p16(out))
    return out


def topk_bf16(values: np.ndarray, k: int) -> Optional[np.ndarray]:
    idx = np.empty(k, dtype=np.int32)
    rc = lib().fwo_topk_bf16(_p16(values), values.size, k, _p32(idx))
    return idx if rc == 0 else None


def route(logits: np.ndarray, k: int):
    idx = np.empty(k, dtype=np.int32)
    scores = np.empty(k, dtype=np.uint16)
    rc = lib().fwo_route(_p16(logits), logits.size, k, _p32(idx), _p16(scores))
    if rc != 0:
        raise ValueError("router received unsupported logits")
    return idx, scores


def equivalent_topk_order(expected, actual, logits: np.ndarray) -> bool:
    e = np.ascontiguousarray(expected, dtype=np.int32)
    a = np.ascontiguousarray(actual, dtype=np.int32)
    if e.size != a.size:
        return False
    return bool(lib().fwo_equivalent_topk_order(_p32(e), _p32(a), e.size, _p16(logits)))


def make_hidden(size: int, spec: dict) -> np.ndarray:
    s = InputSpec(spec["multiplier"], spec["add"], spec["modulus"], spec["center"],
                  spec["divisor"], spec["sparse_stride"])
    out = np.empty(size, dtype=np.uint16)
    if lib().fwo_make_hidden(size, ctypes.byref(s), _p16(out)) != 0:
        raise ValueError("invalid input specification")
    return out


# ---- synthetic data ---------------------------------------------------------

# Tensor ids of the seeded generator; the CUDA generator uses the same ids.
T_ROUTER, T_GATE_UP, T_DOWN, T_SH_GATE, T_SH_UP, T_SH_DOWN, T_SH_GATE_W = range(7)


def synth_scale(std: float) -> float:
    return float(lib().fwo_synth_scale(std))


def synth_bf16(seed: int, tensor: int, start: int, count: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(count, dtype=np.uint16)
    lib().fwo_synth_bf16(seed, tensor, start, count, lib().fwo_synth_scale(std), _p16(out))
    return out


def synth_input(seed: int, rows: int, hidden: int) -> np.ndarray:
    out = np.empty(rows * hidden, dtype=np.uint16)
    lib().fwo_synth_input(seed, rows, hidden, _p16(out))
    return out.reshape(rows, hidden)


def zipf_bias(experts: int) -> np.ndarray:
    out = np.empty(experts, dtype=np.float32)
    lib().fwo_zipf_bias(experts, _pf(out))
    return out


@dataclass
class BlockShape:
    hidden: int
    intermediate: int
    shared_intermediate: int
    experts: int = 512
    top_k: int = 10

    def c(self) -> Shape:
        return Shape(self.hidden, self.intermediate, self.shared_intermediate, self.experts,
                     self.top_k)


class SynthLayer:
    """Host copy of one synthetic layer.  Expert banks are generated lazily,
    per expert, so a CPU run touches only the experts its tokens select."""

    def __init__(self, shape: BlockShape, seed: int, std: float = 0.02, zipf: bool = False):
        self.shape, self.seed, self.std = shape, seed, std
        H, I, Is, E = shape.hidden, shape.intermediate, shape.shared_intermediate, shape.experts
        self.router = synth_bf16(seed, T_ROUTER, 0, E * H, std)
        self.shared_gate = synth_bf16(seed, T_SH_GATE, 0, Is * H, std)
        self.shared_up = synth_bf16(seed, T_SH_UP, 0, Is * H, std)
        self.shared_down = synth_bf16(seed, T_SH_DOWN, 0, H * Is, std)
        self.shared_gate_w = synth_bf16(seed, T_SH_GATE_W, 0, H, std)
        self.bias = zipf_bias(E) if zipf else None
        self.gate_up: dict = {}
        self.down: dict = {}

    def expert(self, e: int):
        H, I = self.shape.hidden, self.shape.intermediate
        if e not in self.gate_up:
            self.gate_up[e] = synth_bf16(self.seed, T_GATE_UP, e * 2 * I * H, 2 * I * H, self.std)
            self.down[e] = synth_bf16(self.seed, T_DOWN, e * H * I, H * I, self.std)
        return self.gate_up[e], self.down[e]

    def ensure(self, experts) -> None:
        for e in sorted(set(int(v) for v in np.asarray(experts).ravel())):
            self.expert(e)

    def _c(self):
        E = self.shape.experts
        gu = (u16p * E)()
        dn = (u16p * E)()
        for e in range(E):
            if e in self.gate_up:
                gu[e] = _p16(self.gate_up[e])
                dn[e] = _p16(self.down[e])
        layer = _Layer(_p16(self.router), gu, dn, _p16(self.shared_gate), _p16(self.shared_up),
                       _p16(self.shared_down), _p16(self.shared_gate_w),
                       _pf(self.bias) if self.bias is not None else None)
        return layer, (gu, dn)


def router(shape: BlockShape, layer: SynthLayer, x: np.ndarray):
    T = x.shape[0]
    x = np.ascontiguousarray(x, dtype=np.uint16)
    idx = np.empty((T, shape.top_k), dtype=np.int32)
    scores = np.empty((T, shape.top_k), dtype=np.uint16)
    logits = np.empty((T, shape.experts), dtype=np.uint16)
    c_layer, keep = layer._c()
    rc = lib().fwo_router(ctypes.byref(shape.c()), ctypes.byref(c_layer), _p16(x), T, _p32(idx),
                          _p16(scores), _p16(logits))
    if rc != 0:
        raise ValueError("oracle router failed")
    return idx, scores, logits


def block(shape: BlockShape, layer: SynthLayer, x: np.ndarray, threads: int = 1,
          taps: bool = False):
    """Whole block for x [T, H]; generates the selected experts first."""
    T = x.shape[0]
    x = np.ascontiguousarray(x, dtype=np.uint16)
    idx, _, _ = router(shape, layer, x)
    layer.ensure(idx)
    return block_resident(shape, layer, x, threads=threads, taps=taps)


def block_resident(shape: BlockShape, layer: SynthLayer, x: np.ndarray, threads: int = 1,
                   taps: bool = False):
    """Whole block; the selected experts must already be generated."""
    T = x.shape[0]
    y = np.empty((T, shape.hidden), dtype=np.uint16)
    idx = np.empty((T, shape.top_k), dtype=np.int32)
    scores = np.empty((T, shape.top_k), dtype=np.uint16)
    c_layer, keep = layer._c()
    tap = None
    tap_arrays = None
    if taps:
        tap_arrays = dict(
            logits=np.empty((T, shape.experts), dtype=np.uint16),
            routed=np.empty((T, shape.hidden), dtype=np.uint16),
            gated_shared=np.empty((T, shape.hidden), dtype=np.uint16),
        )
        tap = _Taps(_p16(tap_arrays["logits"]), _p16(tap_arrays["routed"]),
                    _p16(tap_arrays["gated_shared"]))
    rc = lib().fwo_block(ctypes.byref(shape.c()), ctypes.byref(c_layer), _p16(x), T, _p16(y),
                         _p32(idx), _p16(scores), ctypes.byref(tap) if tap else None, threads)
    if rc != 0:
        raise ValueError(f"oracle block failed ({rc})")
    if taps:
        return y, idx, scores, tap_arrays
    return y, idx, scores


# ---- the reference's own top-k shim (compiled from its source into _ref/) ----

def reference_topk_shim():
    """Return a callable over the reference's native/topk_shim.cpp, or None
    when it was not built (the reference tree is absent)."""
    if not os.path.exists(_SHIM_PATH):
        return None
    L = ctypes.CDLL(_SHIM_PATH)
    fn = L.firewing_torch_topk_bf16
    fn.restype = ctypes.c_bool
    fn.argtypes = [u16p, ctypes.c_size_t, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]

    def call(values: np.ndarray, k: int):
        out = (ctypes.c_size_t * k)()
        ok = fn(_p16(values), values.size, k, out)
        return list(out) if ok else None

    return call


# ---- hyper-connection caller (src/hyper_connection.rs) -----------------------

def inner_square_sum(values: np.ndarray) -> float:
    v = np.ascontiguousarray(values, dtype=np.float32)
    return float(lib().fwo_inner_square_sum(_pf(v), v.size))


def grouped_rms(x: np.ndarray, weight: np.ndarray, hidden: int, eps: float = 1.0e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    out = np.empty_like(x)
    lib().fwo_grouped_rms(_p16(x), _p16(np.ascontiguousarray(weight, dtype=np.uint16)), hidden,
                          x.size // hidden, eps, _p16(out))
    return out


def four_stream_mean(values) -> float:
    v = np.asarray(values, dtype=np.float32)
    return float(lib().fwo_four_stream_mean(_pf(v)))


class HcLayer:
    """Seeded synthetic hyper-connection weights for one layer: hc_norm [4H],
    input_mix_weight_down [LR][4H], input_mix_weight_up [4H][LR],
    block_inject_weight [4][4H]."""

    T_NORM, T_DOWN, T_UP, T_INJECT = 20, 21, 22, 23

    def __init__(self, hidden: int, lowrank: int, seed: int, std: float = 0.02):
        HH = 4 * hidden
        self.hidden, self.lowrank = hidden, lowrank
        self.norm = synth_bf16(seed, self.T_NORM, 0, HH, std)
        self.mix_down = synth_bf16(seed, self.T_DOWN, 0, lowrank * HH, std)
        self.mix_up = synth_bf16(seed, self.T_UP, 0, HH * lowrank, std)
        self.inject = synth_bf16(seed, self.T_INJECT, 0, 4 * HH, std)

    def c(self):
        return _HcLayer(_p16(self.norm), _p16(self.mix_down), _p16(self.mix_up), _p16(self.inject))


def hc_pre(layer: HcLayer, post: np.ndarray):
    """post [T][4H] -> (mixed [T][H], injection weights [T][4])."""
    post = np.ascontiguousarray(post, dtype=np.uint16)
    T, H = post.shape[0], layer.hidden
    mixed = np.empty((T, H), dtype=np.uint16)
    inj = np.empty((T, 4), dtype=np.uint16)
    c = layer.c()
    for t in range(T):
        lib().fwo_hc_pre(_p16(post[t]), ctypes.byref(c), H, layer.lowrank, _p16(mixed[t]), _p16(inj[t]), None)
    return mixed, inj


def hc_post(post: np.ndarray, moe: np.ndarray, inj: np.ndarray) -> np.ndarray:
    post = np.ascontiguousarray(post, dtype=np.uint16)
    moe = np.ascontiguousarray(moe, dtype=np.uint16)
    inj = np.ascontiguousarray(inj, dtype=np.uint16)
    T, H = moe.shape
    out = np.empty_like(post)
    for t in range(T):
        lib().fwo_hc_post(_p16(post[t]), _p16(moe[t]), _p16(inj[t]), H, _p16(out[t]))
    return out
