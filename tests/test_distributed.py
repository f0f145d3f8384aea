"""Sharded summarize on world_size-2 gloo ranks (CPU) equals the single-process summarize.

The two kernel calls (trial analysis and the group bootstrap) are replaced in
both runs by the same deterministic CPU stand-ins, so the test checks exactly
the host logic under test: global duplicate removal, trial and group
sharding, the two exchanges and the summary assembly.
"""
from __future__ import annotations

import hashlib
import math
import multiprocessing as mp
import os
import pickle
import socket
import statistics
import tempfile

import numpy as np
import pytest

from oracle import analysis_oracle as O

WIDTH = 54


def _h(text: str, salt: int = 0) -> int:
    return int(hashlib.sha256(f"{salt}:{text}".encode()).hexdigest()[:12], 16)


def fake_analyze_rows(records, policy, hbm_bandwidth_fraction):
    trials, rows = [], []
    for rec in records:
        h = _h(rec["trial_id"])
        trial = {"trial_id": rec["trial_id"], "valid": h % 9 != 0, "repeat_index": rec["repeat"],
                 "config": rec["config"], "gpu_uuid": "GPU-fake", "workload": rec["workload"],
                 "benchmark_sha256": None, "measurement_stratum": "s", "treatment_design_stratum": "paired",
                 "resource_geometry": {"blocks": 296}, "count_energy_time_alignment_exact": True,
                 "clock_comparison_controlled": True, "diagnostic_only": False, "gpu_name": "B200",
                 "baseline_valid": h % 5 != 0, "operational_idle_increment_eligible": True,
                 "paired_active_reference_eligible": True,
                 "paired_active_reference_protocol": {"order": "AB" if rec["repeat"] % 2 == 0 else "BA"},
                 "paired_active_reference_power_w": 300.0 + h % 17, "hbm_memory_power": None,
                 "target_verified": False, "verified_selection_eligible": False, "ncu_status": "unprofiled",
                 "ncu_utilization_status": "inconclusive",
                 "measurement_diagnostics": {"objectives": {"operational_idle_increment": {"power_w": 1.0 + h % 3},
                                                            "paired_active_reference": {"power_w": 2.0}},
                                             "scope_factors": {"total_over_idle_increment": 1.5 + h % 4}}}
        row = [float(_h(rec["trial_id"], k) % 100_000) / 97.0 for k in range(WIDTH)]
        for k in range(0, WIDTH, 11):
            if _h(rec["trial_id"], 1000 + k) % 4 == 0:
                row[k] = math.nan
        trials.append(trial)
        rows.append(row)
    return trials, np.array(rows, dtype=np.float64).reshape(len(records), WIDTH)


def fake_bootstrap(values, members, seeds, resamples):
    G = len(members)
    med, lo, hi = (np.full((G, values.shape[1]), np.nan) for _ in range(3))
    for g, (rows, seed) in enumerate(zip(members, seeds)):
        for m in range(values.shape[1]):
            vals = [float(values[r, m]) for r in rows if not math.isnan(values[r, m])]
            if vals:
                med[g, m] = statistics.median(vals)
            ci = O.median_ci(vals, seed, resamples)
            if ci:
                lo[g, m], hi[g, m] = ci
    return med, lo, hi


def make_records(n_points=7, repeats=4):
    out = []
    for p in range(n_points):
        for r in range(repeats):
            out.append({"trial_id": f"p{p}-r{r}", "repeat": r, "workload": "tensor",
                        "config": {"point": p, "repeat": r, "blocks": 296}})
    return out


def rank_records(records, rank, world):
    # interleaved ownership plus one duplicate id held by both ranks
    mine = [rec for i, rec in enumerate(records) if i % world == rank]
    return mine + ([dict(records[0])] if rank == world - 1 else [])


def _patch(A):
    A.analyze_rows = fake_analyze_rows
    A.bootstrap_groups = fake_bootstrap


def _worker(rank, world, port, out_path):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from powermodeling_b200 import analysis as A
        from powermodeling_b200.distributed import summarize_sharded
        _patch(A)
        records = rank_records(make_records(), rank, world)
        summary = summarize_sharded(records, resamples=200)
        with open(f"{out_path}.{rank}", "wb") as f:
            pickle.dump(summary, f)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reference_order(world):
    """The concatenation summarize_sharded is defined against: rank 0's records, then rank 1's ..."""
    records = make_records()
    return [rec for r in range(world) for rec in rank_records(records, r, world)]


@pytest.mark.parametrize("world", [2])
def test_sharded_summary_equals_single_process(world, monkeypatch):
    from powermodeling_b200 import analysis as A
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "summary")
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        results = []
        for r in range(world):
            with open(f"{out}.{r}", "rb") as f:
                results.append(pickle.load(f))
    monkeypatch.setattr(A, "analyze_rows", fake_analyze_rows)
    monkeypatch.setattr(A, "bootstrap_groups", fake_bootstrap)
    expected = A.summarize(_reference_order(world), resamples=200)
    assert expected["duplicate_trial_ids_ignored"] == ["p0-r0"]
    assert len(expected["groups"]) == 7
    for got in results:
        assert got == expected


def test_shard_and_ownership_cover_everything_once():
    from powermodeling_b200.distributed import owned_groups, shard_range
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
            owned = sorted(g for r in range(world) for g in owned_groups(n, world, r))
            assert owned == list(range(n))
