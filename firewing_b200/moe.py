"""ctypes binding of libfwmoe (include/fwmoe.h).

Mirrors the reference crate's API for the sparse-MoE block:

* ``MoeBlock`` -- the resident runner (``ExactResidentTop10Runner``,
  src/metal_moe.rs:399-447): install weights once, then run the whole block
  (router -> top-k -> routed SwiGLU experts -> ascending-id bf16 combine ->
  sigmoid-gated shared expert) per call;
* ``linear_bf16`` / ``swiglu_bf16`` / ``route_bf16`` / ``topk_bf16`` -- the
  crate's primitives (src/expert.rs:554-571, src/decoder_layer.rs:278-307,
  native/topk_shim.cpp:18-44) over device buffers.

Errors follow the reference's fail-closed ``Result<_, String>``: every
non-zero status raises ``FwError`` carrying the library's message.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

FW_OK = 0
FW_EINVAL = -1
FW_ECUDA = -2
FW_ENCCL = -3
FW_ETIMEOUT = -4
FW_ENOMEM = -5
FW_ENAN = -6

# expert-parallel transports (fw_moe_ep_set_transport)
EP_TRANSPORT_P2P = 0
EP_TRANSPORT_NCCL = 1

# paths a forward takes (fw_moe_last_path)
PATH_DECODE = 1
PATH_PREFILL = 2

_HERE = os.path.dirname(os.path.abspath(__file__))


def library_path() -> str:
    return os.path.join(_HERE, "libfwmoe.so")


class FwError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"fwmoe error {code}: {message}")
        self.code = code
        self.message = message


class _Config(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("shared_intermediate", ctypes.c_int32),
        ("experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("layers", ctypes.c_int32),
    ]


class _Weights(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "router", "gate_up", "down", "shared_gate", "shared_up", "shared_down", "shared_gate_w",
        "logit_bias")]


_lib = None
vp = ctypes.c_void_p


def library() -> ctypes.CDLL:
    """Load libfwmoe.so (built in-tree by firewing_b200/build.py)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python firewing_b200/build.py` "
            "(there is no CPU fallback)")
    L = ctypes.CDLL(path)
    L.fw_last_error.restype = ctypes.c_char_p
    L.fw_last_error.argtypes = []
    L.fw_moe_create.argtypes = [ctypes.POINTER(_Config), ctypes.c_int, ctypes.POINTER(vp)]
    L.fw_moe_destroy.argtypes = [vp]
    L.fw_moe_load_layer.argtypes = [vp, ctypes.c_int32] + [vp] * 7 + [vp]
    L.fw_moe_synth_layer.argtypes = [vp, ctypes.c_int32, ctypes.c_uint64, ctypes.c_float,
                                     ctypes.c_int32]
    L.fw_moe_forward.argtypes = [vp, ctypes.c_int32, vp, ctypes.c_int32, vp, vp, vp]
    L.fw_moe_forward_async.argtypes = [vp, ctypes.c_int32, vp, ctypes.c_int32, vp, vp, vp, vp]
    L.fw_moe_sync.argtypes = [vp, vp]
    L.fw_moe_set_prefill_min_tokens.argtypes = [vp, ctypes.c_int32]
    L.fw_ep_unique_id.argtypes = [ctypes.c_char_p]
    L.fw_moe_load_hc.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, vp, vp, vp, vp]
    L.fw_moe_forward_hc.argtypes = [vp, ctypes.c_int32, vp, ctypes.c_int32, vp, vp, vp]
    L.fw_moe_forward_hc_async.argtypes = [vp, ctypes.c_int32, vp, ctypes.c_int32, vp, vp, vp, vp]
    L.fw_moe_ep_init.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_char_p]
    L.fw_moe_ep_set_transport.argtypes = [vp, ctypes.c_int32]
    L.fw_moe_set_wait_limit.argtypes = [vp, ctypes.c_uint64]
    L.fw_moe_test_stall.argtypes = [vp]
    L.fw_moe_load_layer_safetensors.argtypes = [vp, ctypes.c_int32, ctypes.c_char_p, ctypes.c_char_p]
    L.fw_moe_load_hc_safetensors.argtypes = [vp, ctypes.c_int32, ctypes.c_char_p, ctypes.c_char_p]
    L.fw_safetensors_tensor_info.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                             ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int32),
                                             ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
    L.fw_moe_get_config.argtypes = [vp, ctypes.POINTER(_Config)]
    L.fw_moe_last_union.argtypes = [vp, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_uint64)]
    L.fw_moe_last_path.argtypes = [vp, ctypes.POINTER(ctypes.c_int32)]
    L.fw_moe_load_expert.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, vp, vp]
    L.fw_moe_load_expert_container.argtypes = [vp, ctypes.c_int32, ctypes.c_char_p, ctypes.c_int32, ctypes.c_int32,
                                               ctypes.POINTER(ctypes.c_int32)]
    L.fw_codec_container_check.argtypes = [ctypes.c_char_p, ctypes.c_int32, ctypes.c_uint64, ctypes.c_int32,
                                           ctypes.POINTER(ctypes.c_int32)]
    L.fw_moe_memory.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64)]
    L.fw_moe_profile.argtypes = [vp, ctypes.c_int32]
    L.fw_moe_profile_read.argtypes = [vp, ctypes.POINTER(ctypes.c_float), ctypes.c_int32]
    L.fw_linear_bf16.argtypes = [vp, vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, vp, vp]
    L.fw_swiglu_bf16.argtypes = [vp, vp, ctypes.c_int64, vp, vp]
    L.fw_add_bf16.argtypes = [vp, vp, ctypes.c_int64, vp, vp]
    L.fw_route_bf16.argtypes = [vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, vp, vp, vp]
    L.fw_moe_forward_noalloc.argtypes = [ctypes.POINTER(_Config), ctypes.POINTER(_Weights), vp,
                                         ctypes.c_int32, vp, vp, vp, vp]
    L.firewing_cuda_topk_bf16.restype = ctypes.c_bool
    L.firewing_cuda_topk_bf16.argtypes = [vp, ctypes.c_size_t, ctypes.c_size_t,
                                          ctypes.POINTER(ctypes.c_size_t)]
    for name in ("fw_moe_create", "fw_moe_destroy", "fw_moe_load_layer", "fw_moe_synth_layer",
                 "fw_moe_forward", "fw_moe_forward_async", "fw_moe_sync", "fw_moe_memory",
                 "fw_moe_profile", "fw_moe_profile_read", "fw_moe_set_prefill_min_tokens",
                 "fw_ep_unique_id", "fw_moe_ep_init", "fw_moe_load_hc", "fw_moe_forward_hc",
                 "fw_moe_forward_hc_async", "fw_moe_load_layer_safetensors", "fw_moe_load_hc_safetensors",
                 "fw_safetensors_tensor_info", "fw_moe_get_config", "fw_moe_last_union", "fw_moe_last_path", "fw_moe_load_expert",
                 "fw_moe_load_expert_container", "fw_codec_container_check",
                 "fw_linear_bf16", "fw_swiglu_bf16", "fw_add_bf16", "fw_route_bf16", "fw_moe_forward_noalloc",
                 "fw_moe_ep_set_transport", "fw_moe_set_wait_limit", "fw_moe_test_stall"):
        getattr(L, name).restype = ctypes.c_int
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc != FW_OK:
        raise FwError(rc, library().fw_last_error().decode("utf-8", "replace"))


def _ptr(a) -> Optional[int]:
    """Address of a numpy array (host) or a torch tensor (host or device)."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        assert a.flags.c_contiguous, "arrays must be C-contiguous"
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        assert a.is_contiguous(), "tensors must be contiguous"
        return a.data_ptr()
    raise TypeError(f"unsupported buffer type {type(a)}")


def _stream(s) -> Optional[int]:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return getattr(s, "cuda_stream", None) or None


@dataclass
class MoeConfig:
    hidden: int = 2048
    intermediate: int = 512
    shared_intermediate: int = 512
    experts: int = 512
    top_k: int = 10
    max_tokens: int = 64
    layers: int = 1

    def c(self) -> _Config:
        return _Config(self.hidden, self.intermediate, self.shared_intermediate, self.experts,
                       self.top_k, self.max_tokens, self.layers)


class MoeBlock:
    """Resident sparse-MoE block runner on one device."""

    def __init__(self, config: MoeConfig, device: int = 0):
        self.config = config
        self.device = device
        h = vp()
        _check(library().fw_moe_create(ctypes.byref(config.c()), device, ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            library().fw_moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> int:
        return self._h.value

    def load_layer(self, layer: int, router, gate_up, down, shared_gate, shared_up, shared_down,
                   shared_gate_w, logit_bias=None) -> None:
        _check(library().fw_moe_load_layer(
            self._h, layer, _ptr(router), _ptr(gate_up), _ptr(down), _ptr(shared_gate),
            _ptr(shared_up), _ptr(shared_down), _ptr(shared_gate_w), _ptr(logit_bias)))

    def synth_layer(self, layer: int, seed: int, std: float = 0.02, zipf: bool = False) -> None:
        _check(library().fw_moe_synth_layer(self._h, layer, seed, std, 1 if zipf else 0))

    def forward(self, layer: int, x: np.ndarray):
        """Host buffers in and out (synchronous): returns (y, topk_idx, scores)."""
        cfg = self.config
        x = np.ascontiguousarray(x, dtype=np.uint16)
        T = x.shape[0]
        y = np.empty((T, cfg.hidden), dtype=np.uint16)
        idx = np.empty((T, cfg.top_k), dtype=np.int32)
        sc = np.empty((T, cfg.top_k), dtype=np.uint16)
        _check(library().fw_moe_forward(self._h, layer, _ptr(x), T, _ptr(y), _ptr(idx), _ptr(sc)))
        return y, idx, sc

    def forward_async(self, layer: int, x, tokens: int, y, topk_idx=None, topk_scores=None,
                      stream=None) -> None:
        """Device buffers (torch tensors or raw addresses), stream-ordered."""
        _check(library().fw_moe_forward_async(self._h, layer, _ptr(x), tokens, _ptr(y),
                                              _ptr(topk_idx), _ptr(topk_scores), _stream(stream)))

    def sync(self, stream=None) -> None:
        _check(library().fw_moe_sync(self._h, _stream(stream)))

    STAGES = ("router", "route", "dispatch", "experts", "combine")

    def ep_init(self, rank: int, world: int, unique_id: bytes, transport: int = EP_TRANSPORT_P2P) -> None:
        """Expert parallelism: this handle holds the experts e with
        e % world == rank and every forward becomes collective over the
        `world` ranks that share `unique_id` (from ep_unique_id on one rank).
        transport: EP_TRANSPORT_P2P (NVLink peer memory, the default) or
        EP_TRANSPORT_NCCL.  Call on every rank before loading layers."""
        if len(unique_id) != 128:
            raise ValueError("unique_id must be 128 bytes")
        _check(library().fw_moe_ep_set_transport(self._h, int(transport)))
        _check(library().fw_moe_ep_init(self._h, int(rank), int(world), bytes(unique_id)))

    def set_wait_limit(self, seconds: float) -> None:
        """Bound of the device-side waits on other CTAs and on peers."""
        _check(library().fw_moe_set_wait_limit(self._h, int(seconds * 1e9)))

    def test_stall(self) -> None:
        """Test hook: the next forward's expert-kernel wait runs out (FW_ETIMEOUT)."""
        _check(library().fw_moe_test_stall(self._h))

    def load_hc(self, layer: int, lowrank: int, hc_norm, mix_down, mix_up, inject) -> None:
        """Hyper-connection weights of one layer (host arrays or device tensors):
        hc_norm [4H], mix_down [lowrank][4H], mix_up [4H][lowrank], inject [4][4H]."""
        keep = [np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a
                for a in (hc_norm, mix_down, mix_up, inject)]
        _check(library().fw_moe_load_hc(self._h, layer, lowrank, *[_ptr(a) for a in keep]))

    def last_union(self) -> dict:
        """Expert union of the last forward: {"distinct_experts": U (routed
        experts streamed on this GPU), "weight_bytes": bytes read}."""
        n, b = ctypes.c_int32(), ctypes.c_uint64()
        _check(library().fw_moe_last_union(self._h, ctypes.byref(n), ctypes.byref(b)))
        return {"distinct_experts": int(n.value), "weight_bytes": int(b.value)}

    def last_path(self) -> int:
        """PATH_DECODE or PATH_PREFILL: the path of this handle's last forward."""
        v = ctypes.c_int32()
        _check(library().fw_moe_last_path(self._h, ctypes.byref(v)))
        return int(v.value)

    def load_expert(self, layer: int, expert: int, gate_up, down) -> None:
        """Replace one routed expert of a loaded layer: gate_up [2I][H] and
        down [H][I] (reference layout), host arrays or device tensors."""
        keep = [np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a for a in (gate_up, down)]
        _check(library().fw_moe_load_expert(self._h, layer, expert, _ptr(keep[0]), _ptr(keep[1])))

    def load_expert_container(self, layer: int, manifest: str, container_layer: int, verify: bool = True) -> int:
        """Experts of `container_layer` from a compressed container (zstd
        frames of byte-shuffled BF16) into `layer`; returns how many."""
        n = ctypes.c_int32()
        _check(library().fw_moe_load_expert_container(self._h, layer, os.fsencode(manifest), container_layer,
                                                      1 if verify else 0, ctypes.byref(n)))
        return int(n.value)

    def load_layer_safetensors(self, layer: int, checkpoint: str, prefix: str) -> None:
        """The block's BF16 tensors under `prefix` (e.g.
        "model.language_model.layers.0.mlp") from a safetensors checkpoint: a
        directory with model.safetensors.index.json, or one file."""
        _check(library().fw_moe_load_layer_safetensors(self._h, layer, os.fsencode(checkpoint),
                                                        prefix.encode()))

    def load_hc_safetensors(self, layer: int, checkpoint: str, prefix: str) -> None:
        """Hyper-connection tensors under `prefix` (e.g.
        "model.language_model.layers.0.mlp_hyper_connection")."""
        _check(library().fw_moe_load_hc_safetensors(self._h, layer, os.fsencode(checkpoint), prefix.encode()))

    def forward_hc(self, layer: int, post: np.ndarray):
        """Attention output post [T][4H] (host) -> (layer output [T][4H],
        top-k ids [T][K], scores [T][K]) through the hyper-connection caller
        and the block."""
        post = np.ascontiguousarray(post, dtype=np.uint16)
        T = post.shape[0]
        out = np.empty_like(post)
        idx = np.empty((T, self.config.top_k), dtype=np.int32)
        sc = np.empty((T, self.config.top_k), dtype=np.uint16)
        _check(library().fw_moe_forward_hc(self._h, layer, _ptr(post), T, _ptr(out), _ptr(idx), _ptr(sc)))
        return out, idx, sc

    def set_prefill_min_tokens(self, min_tokens: int) -> None:
        """Forwards of at least min_tokens tokens (and all above 256) take the
        tensor-core prefill path; narrower ones the bit-exact decode path.
        Under expert parallelism the width is tokens x world.  Default 96
        for shapes with a prefill path."""
        _check(library().fw_moe_set_prefill_min_tokens(self._h, int(min_tokens)))

    def profile(self, enable: bool) -> None:
        _check(library().fw_moe_profile(self._h, 1 if enable else 0))

    def profile_read(self) -> dict:
        """Stage durations (ms) of the last forward while profiling is on."""
        buf = (ctypes.c_float * len(self.STAGES))()
        _check(library().fw_moe_profile_read(self._h, buf, len(self.STAGES)))
        return dict(zip(self.STAGES, [float(v) for v in buf]))

    def memory_bytes(self) -> int:
        v = ctypes.c_uint64()
        _check(library().fw_moe_memory(self._h, ctypes.byref(v)))
        return int(v.value)


def safetensors_tensor_info(file: str, tensor: str) -> dict:
    """Validate a safetensors file as the checkpoint loader does and report
    one tensor: {"dtype", "shape", "offset", "bytes"} (offset within the
    payload).  Raises FwError on any validation failure."""
    L = library()
    dtype = ctypes.create_string_buffer(16)
    shape = (ctypes.c_int64 * 8)()
    rank = ctypes.c_int32()
    offset, nbytes = ctypes.c_uint64(), ctypes.c_uint64()
    _check(L.fw_safetensors_tensor_info(os.fsencode(file), tensor.encode(), dtype, shape, ctypes.byref(rank),
                                        ctypes.byref(offset), ctypes.byref(nbytes)))
    return {"dtype": dtype.value.decode(), "shape": [int(shape[i]) for i in range(rank.value)],
            "offset": int(offset.value), "bytes": int(nbytes.value)}


def codec_container_check(manifest: str, layer: int, source_bytes_per_expert: int, verify: bool = True) -> int:
    """Validate a compressed expert container's manifest and decode (and with
    `verify`, hash-check) the records of `layer` (all when < 0) without a
    GPU; returns the number of records.  Raises FwError on any mismatch."""
    n = ctypes.c_int32()
    _check(library().fw_codec_container_check(os.fsencode(manifest), layer, source_bytes_per_expert,
                                              1 if verify else 0, ctypes.byref(n)))
    return int(n.value)


def ep_owner(expert: int, world: int) -> int:
    """Rank that holds `expert` under expert parallelism (interleaved
    placement: expert e lives on rank e % world, at bank index e // world)."""
    return expert % world


def ep_held_experts(experts: int, world: int, rank: int):
    """Experts held by `rank`, ascending."""
    if experts % world:
        raise ValueError("experts must divide evenly over the ranks")
    return list(range(rank, experts, world))


def ep_combine_row(expert: int, t_local: int, k: int, tokens_local: int, top_k: int, world: int) -> int:
    """Row of the decode combine's receive buffer that holds the weighted
    output of `expert` for the owner's token t_local at top-k position k: the
    rows arrive as one [tokens_local][top_k] block per source rank."""
    return (ep_owner(expert, world) * tokens_local + t_local) * top_k + k


def ep_unique_id() -> bytes:
    """A fresh NCCL communicator id (128 bytes) for MoeBlock.ep_init."""
    buf = ctypes.create_string_buffer(128)
    _check(library().fw_ep_unique_id(buf))
    return buf.raw


def forward_noalloc(config: MoeConfig, weights: dict, x, tokens: int, y, topk_idx=None,
                    topk_scores=None, stream=None) -> None:
    """The block over caller-owned DEVICE buffers with no device allocation
    (fw_moe_forward_noalloc): for callers that cannot cudaMalloc.  `weights`
    maps router, gate_up, down, shared_gate, shared_up, shared_down,
    shared_gate_w and optionally logit_bias to device buffers.  Synchronous."""
    w = _Weights(*[_ptr(weights.get(name)) for name, _ in _Weights._fields_])
    _check(library().fw_moe_forward_noalloc(ctypes.byref(config.c()), ctypes.byref(w), _ptr(x),
                                            tokens, _ptr(y), _ptr(topk_idx), _ptr(topk_scores),
                                            _stream(stream)))


def linear_bf16(w, x, rows: int, cols: int, tokens: int, y, stream=None) -> None:
    _check(library().fw_linear_bf16(_ptr(w), _ptr(x), rows, cols, tokens, _ptr(y), _stream(stream)))


def add_bf16(a, b, n: int, out, stream=None) -> None:
    """out = add_bf16(a, b) for n bf16 elements (device tensors)."""
    _check(library().fw_add_bf16(_ptr(a), _ptr(b), n, _ptr(out), _stream(stream)))


def swiglu_bf16(gate, up, n: int, out, stream=None) -> None:
    _check(library().fw_swiglu_bf16(_ptr(gate), _ptr(up), n, _ptr(out), _stream(stream)))


def route_bf16(logits, tokens: int, experts: int, top_k: int, indices, scores, stream=None) -> None:
    _check(library().fw_route_bf16(_ptr(logits), tokens, experts, top_k, _ptr(indices),
                                   _ptr(scores), _stream(stream)))


def topk_bf16(values: np.ndarray, k: int):
    """Drop-in of firewing_torch_topk_bf16 (host buffers); None on failure."""
    values = np.ascontiguousarray(values, dtype=np.uint16)
    out = (ctypes.c_size_t * k)()
    ok = library().firewing_cuda_topk_bf16(_ptr(values), values.size, k, out)
    return list(out) if ok else None
