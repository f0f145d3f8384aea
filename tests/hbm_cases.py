"""Deterministic inputs for the HBM bandwidth gate (hbm_bandwidth.py:42-125).

``trial_cases()`` yields (record, trial, selected samples, minimum fraction)
and ``group_cases()`` (valid trials carrying their trial records, workload,
minimum fraction), drawn from a seeded generator that mixes valid evidence
with every way it can be missing or wrong: bus widths, window clocks, MIG
modes and their errors, UUIDs, rates, cache policies.
tests/golden/make_hbm_golden.py runs the reference's trial_bandwidth and
group_bandwidth on them; tests/test_hbm.py checks powermodeling_b200.hbm.
"""
from __future__ import annotations

import random

NAN = float("nan")


def _record(rng):
    r = {"cuda_device": {}, "device": {}, "config": {}}
    if rng.random() < 0.9:
        r["cuda_device"]["memory_bus_width_bits"] = rng.choice([8192] * 12 + [8192.0, 8190, 0, -8, None, True, "x", NAN, 4096])
    if rng.random() < 0.2:
        r["cuda_device"]["uuid"] = rng.choice(["GPU-a", "GPU-b", "MIG-1"])
    if rng.random() < 0.15:
        r["device"]["mig_mode"] = rng.choice([None, 0, 1, "enabled", {"current": None}, {"current": 0}, {"current": 1}])
    if rng.random() < 0.3:
        r["device"]["errors"] = {"mig_mode": rng.choice([{"code": 3}, {"type": "NVMLError_NotSupported"}, {"code": 2}])}
    if rng.random() < 0.05:
        r["quality"] = {"mig_active": rng.choice([True, False])}
    if rng.random() < 0.05:
        r["config"]["gpu_uuid"] = rng.choice(["GPU-a", "MIG-x"])
    return r


def _trial(rng):
    t = {"workload": rng.choice(["hbm"] * 9 + ["l2"]),
         "throughput_bytes_s": rng.choice([6e12, 7.9e12, 1e12, 0, -5.0, None, float("inf"), 9e12, 7.0e12])}
    if rng.random() < 0.5:
        t["gpu_uuid"] = rng.choice(["GPU-a", "GPU-b"])
    if rng.random() < 0.5:
        t["experiment_contract"] = {"access": rng.choice(["read", "copy"]), "read_cache_policy": rng.choice(["cg", "cs", "ca"])}
    return t


def _samples(rng):
    if rng.random() < 0.8:
        return [{"memory_clock_mhz": 3996}] * 3
    values = [3996] * 30 + [3996.0, 2000, 0, None, -1, True, NAN, 1e308]
    return [{"memory_clock_mhz": rng.choice(values)} for _ in range(rng.randint(0, 4))]


def trial_cases(n: int = 1500, seed: int = 7):
    rng = random.Random(seed)
    return [(_record(rng), _trial(rng), _samples(rng), rng.choice([0.8, 0.5, 1.0])) for _ in range(n)]


def group_cases(trial_bandwidth, n: int = 600, seed: int = 11):
    """Groups whose trials carry ``hbm_bandwidth`` records made by the given trial_bandwidth."""
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        trials = []
        for _ in range(rng.randint(0, 4)):
            t = _trial(rng)
            t["workload"] = "hbm"
            record, samples = _record(rng), _samples(rng)
            t["hbm_bandwidth"] = trial_bandwidth(record, t, samples, 0.8) if rng.random() < 0.9 else None
            trials.append(t)
        out.append((trials, rng.choice(["hbm", "hbm", "l1"]), rng.choice([0.8, 0.5])))
    return out
