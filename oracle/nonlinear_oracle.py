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


# ---------------------------------------------------------------- count contract
def _count(obj, key, bad):
    v = obj.get(key)
    ok = not isinstance(v, bool) and isinstance(v, (int, float)) and np.isfinite(v) and v >= 0 and v == int(v)
    if not ok:
        bad.add("invalid_nonlinear_count:" + key)
    return v if ok else None


def _mul(*vals):
    if any(v is None for v in vals):
        return None
    out = 1
    for v in vals:
        out *= v
    return out


def count_issues(bench: dict, workload: str) -> list[str]:
    """The reference's nonlinear.count_issues (nonlinear.py:22-128), restated independently of the product."""
    if workload not in FUNCTIONS:
        return []
    import math
    bad: set[str] = set()
    row = workload in ROW_FUNCTIONS
    bpe = 16 if row else 8
    c = lambda key, obj=bench: _count(obj, key, bad)  # noqa: E731

    def eq(name, a, b):
        if a is None or b is None or not math.isclose(a, b, rel_tol=1e-9, abs_tol=1e-6):
            bad.add("nonlinear_count_disagreement:" + name)

    el, ops = c("elements"), c("operations")
    if el is not None and el <= 0:
        bad.add("missing_nonlinear_elements")
    eq("operations_are_elements", ops, el)
    eq("logical_bytes", c("logical_bytes"), _mul(el, bpe))
    w = c("row_width")
    if row:
        if w is None or not 1 <= w <= 65536:
            bad.add("invalid_nonlinear_row_width")
        eq("row_evaluations", c("row_evaluations"), el / w if el is not None and w else None)
    else:
        eq("row_width", w, 0)
        eq("row_evaluations", c("row_evaluations"), 0)
    blocks, ws, it, adm = c("blocks"), c("working_set_bytes"), c("iterations_per_launch"), c("admitted_blocks")
    qg = bench.get("math_implementation") == "cuda_fp32_q_grid_v2" or \
        bench.get("kernel_implementation_version") == "fp32_complete_nonlinear_q_grid_v2"
    launches = bl = q = None
    if qg:
        if (bench.get("math_implementation"), bench.get("kernel_implementation_version")) != \
                ("cuda_fp32_q_grid_v2", "fp32_complete_nonlinear_q_grid_v2"):
            bad.add("unsupported_nonlinear_q_grid_implementation")
        if bench.get("block_completion_count_source") != "synchronized_completed_launches":
            bad.add("unsupported_nonlinear_block_completion_count_source")
        q, th, launches = c("input_elements"), c("threads"), c("kernel_launches")
        if "batch_launches" in bench:
            bl = c("batch_launches")
            if not bl:
                bad.add("invalid_nonlinear_batch_launches")
        if "batches" in bench:
            eq("completed_batch_kernel_launches", launches, _mul(c("batches"), bl))
        if ws is None or ws <= 0 or ws % 4:
            bad.add("invalid_nonlinear_input_word_alignment")
        eq("input_elements", q, ws / 4 if ws is not None else None)
        if q is None or q <= 0 or (w and row and q % w):
            bad.add("incomplete_nonlinear_input_or_row")
        if th is None or not 32 <= th <= 1024 or th % 32:
            bad.add("invalid_nonlinear_threads")
        mode = bench.get("grid_mode")
        if mode not in ("auto", "fixed"):
            bad.add("invalid_nonlinear_grid_mode")
        elif mode == "auto" and q and th and (not row or w):
            eq("auto_grid_blocks", blocks, q / w if row else math.ceil(q / th))
        if not blocks or blocks > 1000000 or not it or not launches:
            bad.add("missing_nonlinear_execution_counts")
        if launches is not None and blocks is not None:
            eq("completed_launch_admissions", adm, launches * blocks)
        eq("completed_launch_elements", el, _mul(launches, q, it))
    elif blocks and ws and it and adm:
        eq("admission_elements", el, adm * (ws / 4 / blocks) * it)
        if ws % (4 * blocks * (w if row and w else 1)):
            bad.add("incomplete_nonlinear_block_slice_or_row")
    else:
        bad.add("missing_nonlinear_execution_counts")
    if bench.get("math_implementation") not in ("cuda_fp32_standard_streaming_v1", "cuda_fp32_q_grid_v2") \
            or bench.get("input_precision") != "fp32":
        bad.add("unsupported_nonlinear_math_contract")
    if workload == "rmsnorm" and (bench.get("rms_epsilon") != 1e-5 or bench.get("affine_gamma") is not True):
        bad.add("unsupported_rmsnorm_definition")
    if (bench.get("sanity") or {}).get("numerical_validation_passed") is not True:
        bad.add("nonlinear_numerical_validation_failed_or_missing")
    chk = (bench.get("numerical_validation") or {}).get("checked_values")
    if isinstance(chk, bool) or not isinstance(chk, (int, float)) or not np.isfinite(chk) or chk <= 0:
        bad.add("missing_nonlinear_numerical_reference_checks")
    epochs = bench.get("measure_epochs")
    if not isinstance(epochs, list) or not epochs:
        bad.add("missing_nonlinear_measure_epochs")
        return sorted(bad)
    for ep in epochs:
        if not isinstance(ep, dict):
            bad.add("invalid_nonlinear_epoch")
            continue
        e = _count(ep, "elements", bad)
        eq("epoch_operations_are_elements", _count(ep, "operations", bad), e)
        eq("epoch_logical_bytes", _count(ep, "logical_bytes", bad), _mul(e, bpe))
        eq("epoch_rows", _count(ep, "row_evaluations", bad), e / w if e is not None and w and row else 0)
        if qg:
            el_ = _count(ep, "kernel_launches", bad)
            if "batches" in ep:
                eq("epoch_completed_batch_kernel_launches", el_, _mul(_count(ep, "batches", bad), bl))
            eq("epoch_completed_launch_admissions", _count(ep, "admitted_blocks", bad), _mul(el_, blocks))
            eq("epoch_completed_launch_elements", e, _mul(el_, q, it))
        if ep.get("counts_exact") is not True:
            bad.add("inexact_nonlinear_measure_epoch")
    tot = lambda k: sum(ep.get(k, 0) for ep in epochs if isinstance(ep, dict) and isinstance(ep.get(k), (int, float)))  # noqa: E731
    eq("epoch_total_elements", tot("elements"), el)
    if qg:
        eq("epoch_total_kernel_launches", tot("kernel_launches"), launches)
    return sorted(bad)
