"""The native record assembly helpers (_recordnative) against their Python statements.

fold: the group diagnostics' fold (trial_report._fold) on nested repeat diagnostics with
every kind of leaf, missing keys, None repeats and values that take the Python path.
phase_dicts: analysis._phase_dict over phase rows with random values, NaNs and flag words.
measurement_diagnostics: trial_report.measurement_diagnostics over randomized trial results of
every workload class, odd value types, epochs with and without counter readbacks, and a bench
that is not a dict.
sorted_json: json.dumps(sort_keys=True, separators=(",", ":")) on randomized nested values.
"""
from __future__ import annotations

import json
import math
import random

import numpy as np
import pytest

from powermodeling_b200 import _native as N
from powermodeling_b200 import analysis as A
from powermodeling_b200 import trial_report as TR


def _same(a, b) -> bool:
    """Equal values of equal types, key order included (NaN equals NaN)."""
    if type(a) is not type(b):
        return False
    if isinstance(a, dict):
        return list(a) == list(b) and all(_same(a[k], b[k]) for k in a)
    if isinstance(a, list):
        return len(a) == len(b) and all(_same(x, y) for x, y in zip(a, b))
    if isinstance(a, float) and math.isnan(a) and math.isnan(b):
        return True
    return a == b


class Weird(float):
    """A float subclass: the fold hands such values to the Python statement."""


def _leaf(rng: random.Random):
    kind = rng.randrange(11)
    if kind == 0:
        return None
    if kind == 1:
        return rng.random() < 0.7
    if kind == 2:
        return rng.choice(["pass", "fail", "inconclusive"])
    if kind == 3:
        return rng.randrange(-5, 50)
    if kind == 4:
        return rng.choice([float("nan"), float("inf"), -0.0, 0.0])
    if kind == 5:
        return [rng.choice(["a", "b", "c", "d"]) for _ in range(rng.randrange(4))]
    if kind == 6:
        return [{"x": rng.randrange(3)}] if rng.random() < 0.5 else [1, "a"]
    if kind == 7:
        return Weird(rng.uniform(0, 10))
    return rng.uniform(-1e3, 1e3)


def _tree(rng: random.Random, depth: int, keys: list[str]):
    if depth == 0 or rng.random() < 0.25:
        return _leaf(rng)
    return {k: _tree(rng, depth - 1, keys) for k in rng.sample(keys, rng.randrange(1, len(keys)))}


def test_fold_equals_python_statement():
    native = TR._record_native()
    rng = random.Random(7)
    keys = [f"k{i}" for i in range(7)]
    for case in range(400):
        repeats = rng.randrange(1, 6)
        template = _tree(rng, 3, keys)
        values = []
        for _ in range(repeats):
            if rng.random() < 0.1:
                values.append(None)
                continue
            # repeats share their shape and mostly their kinds, as real diagnostics do
            v = json.loads(json.dumps(template, default=float)) if isinstance(template, dict) else template
            values.append(_tree(rng, 3, keys) if rng.random() < 0.3 else _perturb(rng, v))
        assert _same(native.fold(values, TR._fold), TR._fold(values)), f"case {case}"


def _perturb(rng, v):
    if isinstance(v, dict):
        out = {k: _perturb(rng, x) for k, x in v.items() if rng.random() > 0.1}
        if rng.random() < 0.2:
            out["extra"] = _leaf(rng)
        return out
    if isinstance(v, float):
        return v * rng.uniform(0.5, 2.0) if math.isfinite(v) else v
    if isinstance(v, bool) or v is None:
        return v if rng.random() < 0.8 else _leaf(rng)
    return v


def test_fold_edge_cases():
    native = TR._record_native()
    cases = [[], [None], [None, None], [True, True], [True, None], [1, 2.5, None, True], [-0.0, 0.0],
             [0.0, -0.0], [2 ** 80, 1], ["s", 1.0], [[], ["a"], ["a", "b"]], [{"a": 1}, None, {"b": [True]}],
             [{"a": {"b": 1.0}}, {"a": None}], [float("nan"), float("inf")], [Weird(1.0), 2.0]]
    for values in cases:
        assert _same(native.fold(values, TR._fold), TR._fold(values)), values
    with pytest.raises(OverflowError):
        native.fold([10 ** 400, 1.0], TR._fold)


def _phase_views(rng: np.random.Generator, n_trials: int):
    views = A._Views(n_trials)
    views.phase_out[:] = rng.uniform(-1e3, 1e3, views.phase_out.size)
    views.phase_out[rng.random(views.phase_out.size) < 0.2] = np.nan
    samples, distinct = A._po_names()["SAMPLES"], A._po_names()["DISTINCT_POWER"]
    rows = views.phase_out.reshape(-1, views.PO)
    rows[:, samples] = rng.integers(0, 400, len(rows))
    rows[:, distinct] = rng.integers(0, 50, len(rows))
    views.phase_flags[:] = rng.integers(0, 2 ** 31, views.phase_flags.size, dtype=np.int64).astype(np.uint32)
    # mostly computed phases: clear the missing and invalid-window bits of most slots
    missing, invalid, _, _ = A._pf_bits()
    keep = rng.random(views.phase_flags.size) < 0.8
    views.phase_flags[keep] &= np.uint32(~((1 << missing) | (1 << invalid)) & 0xFFFFFFFF)
    return views


def test_phase_dicts_equal_python_statement():
    if not N.LIBRARY.exists():
        pytest.skip("libpmb200 not built")
    rng = np.random.default_rng(11)
    views = _phase_views(rng, 40)
    policy = A.AnalysisPolicy()
    native = A._phase_dicts(views)
    assert len(native) == 40 * N.PM_PHASES
    for slot, got in enumerate(native):
        name = N.PHASE_NAMES[slot % N.PM_PHASES]
        po = views.phase_out[slot * views.PO:(slot + 1) * views.PO]
        want = A._phase_dict(name, po, int(views.phase_flags[slot]), policy)
        assert _same(got, want), (slot, got, want)


def _diagnostic_case(rng: random.Random):
    from types import MappingProxyType
    workloads = ["hbm", "l1", "tensor", "gemm", "sfu_ex2", "softmax", "exp", "control", None]
    numeric = lambda: rng.choice([None, rng.uniform(-5, 500), rng.randrange(0, 10 ** 6), float("nan"), float("inf"),
                                  True, "12.5", "x", 0.0, -0.0])
    result = {"workload": rng.choice(workloads)}
    for key in ("throughput_bytes_s", "counted_measure_logical_bytes", "throughput_ops_s", "counted_measure_operations",
                "duration_s", "board_power_w", "idle_power_w", "active_reference_power_w",
                "paired_active_reference_power_w", "operational_idle_increment_power_w", "integrated_power_energy_j",
                "energy_counter_j", "total_energy_j", "operational_idle_increment_energy_j",
                "paired_active_reference_energy_j", "total_pj_per_logical_bit", "total_pj_per_flop",
                "operational_idle_increment_pj_per_instruction", "paired_active_reference_pj_per_element"):
        if rng.random() < 0.85:
            result[key] = numeric()
    for key in ("count_energy_time_alignment_exact", "valid", "operational_idle_increment_eligible",
                "paired_active_reference_eligible", "target_verified", "baseline_valid"):
        if rng.random() < 0.9:
            result[key] = rng.choice([True, False, 1, None])
    for key in ("flop_count_convention", "energy_source", "sfu_contract", "sfu_reference_delta_diagnostics"):
        if rng.random() < 0.7:
            result[key] = rng.choice(["text", None, {"a": 1}])
    if rng.random() < 0.7:
        result["issues"] = ["a", "b"][:rng.randrange(3)]
    if rng.random() < 0.7:
        result["baseline_issues"] = []
    bench = {k: rng.choice(["u", 3, None, {"k": [1]}]) for k in (
        "operation_unit", "kernel_resources", "auxiliary_work", "execution_diagnostics", "kernel_implementation_version",
        "memory_accesses_per_thread_iteration", "grid_mode", "active_sm_ids", "duration_scope") if rng.random() < 0.6}
    for key in ("host_duration_s", "duration_s", "mean_batch_duration_s"):
        if rng.random() < 0.7:
            bench[key] = numeric()
    if rng.random() < 0.2:
        bench = MappingProxyType(bench)
    epochs = []
    t = rng.uniform(0, 5)
    for _ in range(rng.randrange(0, 6)):
        start = t + rng.uniform(0, 0.01)
        t = start + rng.uniform(0.001, 0.2)
        epoch = {"start_s": start, "end_s": t}
        if rng.random() < 0.8:
            epoch["counter_readback_ns"] = rng.choice([rng.randrange(0, 50000), -5, None, 12.5, float("nan")])
        epochs.append(epoch)
    return result, bench, epochs


def test_measurement_diagnostics_equal_python_statement():
    from powermodeling_b200.pack import MEMORY_WORKLOADS, NONLINEAR_WORKLOADS, SFU_WORKLOADS, TENSOR_WORKLOADS
    native = TR._record_native()
    rng = random.Random(3)
    for case in range(600):
        result, bench, epochs = _diagnostic_case(rng)
        want = TR.measurement_diagnostics(result, bench, epochs)
        got = native.measurement_diagnostics(result, bench, epochs, MEMORY_WORKLOADS, TENSOR_WORKLOADS, SFU_WORKLOADS,
                                             NONLINEAR_WORKLOADS, sum)
        assert _same(got, want), (case, result, bench, epochs)
        # values read from the records are the records' own objects
        assert got["quality"]["issues"] is result.get("issues", got["quality"]["issues"])


class Flag(int):
    pass


def _json_value(rng: random.Random, depth: int):
    kind = rng.randrange(12 if depth < 4 else 8)
    if kind == 0:
        return None
    if kind == 1:
        return rng.random() < 0.5
    if kind == 2:
        return rng.randrange(-10 ** 30, 10 ** 30)
    if kind == 3:
        return rng.choice([rng.uniform(-1e6, 1e6), 1e-320, -0.0, float("nan"), float("inf"), -float("inf"), 0.1])
    if kind == 4:
        return "".join(rng.choice(["a", "Z", " ", '"', "\\", "\n", "\t", "\x01", "\x7f", "é", "☃", "\U0001F600", "/"])
                       for _ in range(rng.randrange(8)))
    if kind == 5:
        return Flag(rng.randrange(5))
    if kind == 6:
        return rng.choice(["gpu", "hbm", ""])
    if kind == 7:
        return rng.uniform(0, 1)
    if kind in (8, 9):
        return [_json_value(rng, depth + 1) for _ in range(rng.randrange(4))] if kind == 8 else \
            tuple(_json_value(rng, depth + 1) for _ in range(rng.randrange(3)))
    keys = rng.choice([["b", "a", "c", "aa", "B"], [3, 1, 2], [1.5, -2.0, 0.25], [True, None]])
    return {k: _json_value(rng, depth + 1) for k in rng.sample(keys, rng.randrange(len(keys) + 1))}


def test_sorted_json_equals_json_dumps():
    native = TR._record_native()
    rng = random.Random(19)
    for case in range(2000):
        value = _json_value(rng, 0)
        try:
            want = json.dumps(value, sort_keys=True, separators=(",", ":"))
        except TypeError:                    # keys that do not sort together: both refuse
            with pytest.raises(TypeError):
                native.sorted_json(value)
            continue
        assert native.sorted_json(value) == want, case
    for bad in ({1: 1, "a": 2}, {(1,): 2}, {"a": object()}, [{1, 2}], {"a": b"x"}):
        with pytest.raises(TypeError):
            json.dumps(bad, sort_keys=True, separators=(",", ":"))
        with pytest.raises(TypeError):
            native.sorted_json(bad)
