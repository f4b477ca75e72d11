"""Seeded synthetic inputs for the benchmark configurations.

The benchmark configurations name synthetic data (no checkpoint or dataset):
hidden states are N(0,1)-like rows, RMS-normalised, in bf16.  Each element is
output i of a SplitMix64 stream (Steele, Lea, Flood 2014) keyed by the seed,
summed as four 16-bit uniforms (Irwin-Hall, n = 4), scaled in f32; each row is
divided by sqrt(mean(x^2) + 1e-6) computed in f64 with a sequential sum, then
rounded to bf16 with the reference's RNE formula.  Weights use the same
stream definition on the device (fw_moe_synth_layer).
"""
from __future__ import annotations

import numpy as np

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
INPUT_TENSOR_ID = 0x1000


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def stream_key(seed: int, tensor: int) -> np.uint64:
    with np.errstate(over="ignore"):
        a = _mix64(np.array([np.uint64(seed) + _GAMMA], dtype=np.uint64))[0]
        b = a + np.uint64(tensor) * _GAMMA + _GAMMA
        return _mix64(np.array([b], dtype=np.uint64))[0]


def irwin_hall(key: np.uint64, start: int, count: int) -> np.ndarray:
    """Integer Irwin-Hall(4) samples i = start..start+count-1 (int32)."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + count + 1, dtype=np.uint64)
        h = _mix64(key + i * _GAMMA)
    parts = [(h >> np.uint64(s)) & np.uint64(0xFFFF) for s in (0, 16, 32, 48)]
    return (sum(p.astype(np.int64) for p in parts) - 131070).astype(np.int32)


def scale_for(std: float) -> np.float32:
    return np.float32(std / np.sqrt((65536.0 * 65536.0 - 1.0) / 3.0))


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def synth_input(seed: int, rows: int, hidden: int) -> np.ndarray:
    """[rows, hidden] bf16 bit patterns."""
    key = stream_key(seed, INPUT_TENSOR_ID)
    s = irwin_hall(key, 0, rows * hidden).reshape(rows, hidden)
    v = s.astype(np.float32) * scale_for(1.0)
    sq = np.cumsum(v.astype(np.float64) ** 2, axis=1)[:, -1]
    inv = 1.0 / np.sqrt(sq / hidden + 1e-6)
    return f32_to_bf16((v.astype(np.float64) * inv[:, None]).astype(np.float32))


def zipf_bias(experts: int) -> np.ndarray:
    """Router logit bias 0.5*ln(rank^-1.1), rank = e + 1 (f32)."""
    e = np.arange(1, experts + 1, dtype=np.float64)
    return (0.5 * np.log(e ** -1.1)).astype(np.float32)
