"""CPU oracle of the streaming nonlinear workloads (test infrastructure only).

Only the tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
use this module, as the checker; nothing on the product path imports it.

Restates, in numpy:
* the input and gamma fill of cuda/nonlinear.cuh:5-14 (``init_nonlinear``):
  w = random_word(i ^ seed) & 0xffff (random_word: gpu_bench.cu:277-282, the
  splitmix64 finaliser truncated to 32 bits); input x = (int(w) - 32768) /
  8192 + shift, gamma = 0.75 + w / 131072.  Every value is exact in fp32;
* the CPU double reference of ``check_nonlinear`` (nonlinear.cuh:97-143):
  exp, tanh, x / (1 + exp(-x)); softmax exp(x - max) / sum; RMSNorm
  x / sqrt(sum x^2 / width + 1e-5f) * gamma, accumulated in double;
* its acceptance rule |y - e| <= 2e-6 + 2e-4 |e| (nonlinear.cuh:113-114), the
  softmax row-sum rule |sum y - 1| <= 2e-4 (nonlinear.cuh:139), the sampled
  item positions (nonlinear.cuh:119-121) and the output-bit checksum
  h = h * 1315423911 + bits (nonlinear.cuh:115-116).
Parity is pinned by the reference's own powerbench (built from its sources)
on the GPU: the pointwise checksums must match it bit for bit.
"""
from __future__ import annotations

import numpy as np

FUNCTIONS = ("exp", "tanh", "silu", "softmax", "rmsnorm")
ROW_FUNCTIONS = ("softmax", "rmsnorm")
RMS_EPSILON_F32 = float(np.float32(1e-5))
MASK64 = (1 << 64) - 1


def random_words(index: np.ndarray) -> np.ndarray:
    """random_word(i) for an array of uint64 i (gpu_bench.cu:277-282)."""
    x = index.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15)
    with np.errstate(over="ignore"):
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return (x ^ (x >> np.uint64(31))).astype(np.uint32)


def fill(n: int, seed: int, shift: float = 0.0, gamma: bool = False) -> np.ndarray:
    """init_nonlinear (nonlinear.cuh:5-14) for elements 0..n-1, as float32."""
    i = np.arange(n, dtype=np.uint64) ^ np.uint64(seed & MASK64)
    bits = (random_words(i) & np.uint32(0xFFFF)).astype(np.int64)
    if gamma:
        return (np.float32(0.75) + bits.astype(np.float32) / np.float32(131072.0)).astype(np.float32)
    return ((bits - 32768).astype(np.float32) / np.float32(8192.0) + np.float32(shift)).astype(np.float32)


def workload_inputs(function: str, n: int, seed: int, width: int = 0):
    """The powerbench arm's input and gamma (gpu_bench.cu:712-716: softmax logits shifted by 100)."""
    x = fill(n, seed, 100.0 if function == "softmax" else 0.0)
    g = fill(width if function == "rmsnorm" else 1, seed ^ 12345, 0.0, gamma=True)
    return x, g


def expected(function: str, x: np.ndarray, gamma: np.ndarray | None = None, width: int = 0) -> np.ndarray:
    """check_nonlinear's double reference for every element (nonlinear.cuh:123-138)."""
    v = x.astype(np.float64)
    if function == "exp":
        return np.exp(v)
    if function == "tanh":
        return np.tanh(v)
    if function == "silu":
        return v / (1.0 + np.exp(-v))
    rows = v.reshape(-1, width)
    if function == "softmax":
        e = np.exp(rows - rows.max(axis=1, keepdims=True))
        return (e / e.sum(axis=1, keepdims=True)).reshape(-1)
    ss = (rows * rows).sum(axis=1, keepdims=True)
    return (rows / np.sqrt(ss / width + RMS_EPSILON_F32) * gamma[:width].astype(np.float64)).reshape(-1)


def within_tolerance(actual: np.ndarray, reference: np.ndarray) -> np.ndarray:
    """nonlinear.cuh:113-114 per element: finite and |y - e| <= 2e-6 + 2e-4 |e|."""
    a = actual.astype(np.float64)
    return np.isfinite(a) & np.isfinite(reference) & (np.abs(a - reference) <= 2e-6 + 2e-4 * np.abs(reference))


def softmax_rows_sum_to_one(actual: np.ndarray, width: int) -> np.ndarray:
    return np.abs(actual.astype(np.float64).reshape(-1, width).sum(axis=1) - 1.0) <= 2e-4


def sample_items(items: int) -> list[int]:
    """Checked item positions: first, middle, last and evenly spread, at most eight (nonlinear.cuh:119-121)."""
    samples = min(items, 8)
    return [0 if samples == 1 else items // 2 if k == samples // 2 else k * (items - 1) // (samples - 1)
            for k in range(samples)]


def sample_checksum(function: str, output: np.ndarray, width: int = 0) -> int:
    """The record's checksum over the sampled outputs of one check pass (nonlinear.cuh:115-116)."""
    w = width if function in ROW_FUNCTIONS else 1
    bits = output.astype(np.float32).view(np.uint32)
    h = 0
    for item in sample_items(output.size // w):
        for b in bits[item * w:(item + 1) * w]:
            h = (h * 1315423911 + int(b)) & MASK64
    return h
