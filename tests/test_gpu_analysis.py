"""GPU parity: libpmb200's analysis against the reference's outputs and the oracle."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import close, diff, load_golden
from oracle import analysis_oracle as O
from trial_builders import scenarios
from tests.golden.make_golden import TRIAL_KEYS, PHASE_KEYS, records_digest

pytestmark = pytest.mark.gpu

# Floating tolerance: 1e-6 relative for energies and pJ/op.
REL = 1e-6
EXACT_KEYS = ("total_energy_j", "integrated_power_energy_j", "energy_counter_j", "board_power_w", "idle_power_w",
              "incremental_energy_j", "pj_per_op", "throughput_ops_s", "paired_active_reference_power_w")


@pytest.fixture(scope="module")
def golden_trials():
    return {c["name"]: c for c in load_golden("analysis_trials.json.gz")["cases"]}


@pytest.mark.parametrize("name,record,policy", scenarios(), ids=[s[0] for s in scenarios()])
def test_trial_matches_reference(gpu_ready, golden_trials, name, record, policy):
    from powermodeling_b200.analysis import analyze_trial
    case = golden_trials[name]
    assert case["digest"] == records_digest([record])
    got = analyze_trial(record, policy)
    expected = case["expected"]
    problems = diff(expected, got, TRIAL_KEYS, rel=REL)
    for phase, stats in expected["phases"].items():
        problems += [f"{phase}.{p}" for p in diff(stats, got["phases"].get(phase, {}), PHASE_KEYS, rel=REL)]
    assert not problems, problems
    # The energy integrals follow CPython's arithmetic exactly.
    for key in EXACT_KEYS:
        if key in expected:
            assert close(expected[key], got.get(key), rel=0.0), (key, expected[key], got.get(key))


@pytest.mark.parametrize("name,record,policy", scenarios(), ids=[s[0] for s in scenarios()])
def test_whole_trial_dict_matches_reference(gpu_ready, name, record, policy):
    """Every field of the reference's analyze_trial result (tests/golden/trial_reports.json.gz)."""
    import json
    from powermodeling_b200.analysis import analyze_trial
    case = next(c for c in load_golden("trial_reports.json.gz") if c["name"] == name)
    assert case["digest"] == records_digest([record])
    got = json.loads(json.dumps(analyze_trial(record, policy)))
    problems = _differences(case["expected"], got)
    assert not problems, problems[:8]


def test_sweep_groups_match_reference(gpu_ready):
    from powermodeling_b200.analysis import group_key, summarize, METRICS
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    for sweep in load_golden("analysis_sweeps.json.gz")["sweeps"]:
        shape = SweepShape(**{k: tuple(v) if isinstance(v, list) else v for k, v in sweep["shape"].items()})
        records = make_sweep(shape, sweep["seed"])
        summary = summarize(records, policy=ANALYSIS_POLICY)
        assert [group_key(t) for t in summary["trials"]] == sweep["group_keys"]
        assert len(summary["groups"]) == len(sweep["groups"])
        for got, exp in zip(summary["groups"], sweep["groups"]):
            assert got["group_id"] == exp["group_id"] and got["valid_repeats"] == exp["valid_repeats"]
            for metric in METRICS:
                assert close(exp["medians"][metric], got[metric], rel=0.0), (metric, exp["medians"][metric], got[metric])
                assert close(exp["ci95"][metric], got["ci95"][metric], rel=0.0), (metric, exp["ci95"][metric], got["ci95"][metric])
            assert got["paired_reference_order_counts"] == exp["paired_reference_order_counts"]
            assert got["paired_active_reference_eligible"] == exp["paired_active_reference_eligible"]
            assert close(exp["paired_reference_order_effect_power_w"], got["paired_reference_order_effect_power_w"], rel=0.0)


def test_median_ci_matches_reference_at_1000_and_10000_draws(gpu_ready):
    from powermodeling_b200.analysis import median_ci
    for case in load_golden("median_ci.json.gz")["cases"]:
        assert median_ci(case["values"], case["seed"]) == case["ci_1000"], case
        assert median_ci(case["values"], case["seed"], 10000) == case["ci_10000"], case


def test_resample_index_stream_is_bit_exact(gpu_ready):
    for s in load_golden("median_ci.json.gz")["streams"]:
        rows = gpu_ready.resample_indices(s["seed"], s["n"], len(s["rows"]))
        assert rows.tolist() == s["rows"]


def test_full_size_sweep_against_oracle(gpu_ready):
    """64 points x 4 repeats, B = 10 000: trial numbers for every trial, CIs for a sample of groups."""
    from powermodeling_b200.analysis import METRICS, summarize
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(), seed=0)
    summary = summarize(records, policy=ANALYSIS_POLICY, resamples=10000)
    assert len(summary["trials"]) == 256 and len(summary["groups"]) == 64
    for record, trial in zip(records, summary["trials"]):
        expected = O.analyze(record, ANALYSIS_POLICY)
        assert trial["valid"]
        assert not diff(expected, trial, ("total_energy_j", "board_power_w", "idle_power_w", "pj_per_op",
                                          "paired_active_reference_pj_per_flop", "throughput_ops_s"), rel=0.0)
    for g in summary["groups"][:3]:
        members = [summary["trials"][records.index(next(r for r in records if r["trial_id"] == tid))] for tid in g["trial_ids"]]
        seed = int(g["group_id"], 16)
        for metric in METRICS:
            vals = [v for t in members if (v := O.num(t.get(metric))) is not None]
            assert g["ci95"][metric] == O.median_ci(vals, seed, 10000), metric


def test_host_staging_rejects_unsorted_samples_then_recovers(gpu_ready):
    """The staged host path checks sample order while copying; an error leaves the workspace reusable."""
    from powermodeling_b200 import _native as N
    from powermodeling_b200 import analysis as A
    from powermodeling_b200.pack import trials_struct
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(points=3, repeats=4), seed=21)
    packed, _, _ = A.prepare(records)
    policy = A.AnalysisPolicy(**ANALYSIS_POLICY).native()
    t_s = packed.arrays["t_s"]
    offsets = packed.arrays["phase_offsets"]
    slot = 7
    i = int(offsets[slot]) + 3
    good = A._Views(packed.n_trials)
    assert N.library().pm_analyze_trials(trials_struct(packed), policy, good.struct()) == 0
    t_s[i], t_s[i + 1] = t_s[i + 1], t_s[i]
    bad = A._Views(packed.n_trials)
    rc = N.library().pm_analyze_trials(trials_struct(packed), policy, bad.struct())
    assert rc == -1 and f"slot {slot}" in N.last_error()   # PM_E_INVALID
    t_s[i], t_s[i + 1] = t_s[i + 1], t_s[i]
    again = A._Views(packed.n_trials)
    assert N.library().pm_analyze_trials(trials_struct(packed), policy, again.struct()) == 0
    assert np.array_equal(np.nan_to_num(good.trial_out), np.nan_to_num(again.trial_out))


@pytest.mark.parametrize("arm_s", [7.0, 15.0, 26.0], ids=["P1024", "P2048", "P4096-global-scratch"])
def test_long_phases_match_oracle(gpu_ready, arm_s):
    """Phases of ~700, ~1500 and ~2600 samples: every sort width of the analysis kernel."""
    from powermodeling_b200.analysis import analyze_trials
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(points=1, repeats=2, arm_s=arm_s, epochs_per_arm=int(arm_s)), seed=9)
    got = analyze_trials(records, ANALYSIS_POLICY)
    for record, trial in zip(records, got):
        expected = O.analyze(record, ANALYSIS_POLICY)
        problems = diff(expected, trial, TRIAL_KEYS, rel=0.0)
        for phase, stats in expected["phases"].items():
            problems += [f"{phase}.{p}" for p in diff(stats, trial["phases"].get(phase, {}), PHASE_KEYS, rel=0.0)]
        assert not problems, problems


@pytest.mark.parametrize("members", [4, 5, 8, 9, 16, 24, 32])
def test_bootstrap_mixed_member_counts_match_oracle(gpu_ready, members):
    """Metrics that lose members to NaN: the prepared draws serve count == members, fresh draws the rest.

    Power-of-two groups (4, 8, 16, 32) take the draw pass whose twist stores the indices itself; the
    others convert word pairs."""
    import hashlib
    import statistics
    from powermodeling_b200.analysis import bootstrap_groups
    rng = np.random.default_rng(members)
    G, M = 6, 12
    values = rng.normal(100, 10, size=(G * members, M)).round(3)
    for g in range(G):
        for m in range(M):
            drop = [0, 1, 3, members - 2][m % 4]
            values[g * members + rng.choice(members, size=drop, replace=False), m] = np.nan
    groups = [list(range(g * members, (g + 1) * members)) for g in range(G)]
    seeds = [int(hashlib.sha256(f"mixed-{members}-{g}".encode()).hexdigest()[:16], 16) for g in range(G)]
    med, lo, hi = bootstrap_groups(values, groups, seeds, 1000)
    for g in range(G):
        for m in range(M):
            vals = [float(v) for v in values[groups[g], m] if not np.isnan(v)]
            ci = O.median_ci(vals, seeds[g], 1000)
            got = None if np.isnan(lo[g, m]) else [float(lo[g, m]), float(hi[g, m])]
            assert got == ci, (g, m, len(vals), got, ci)
            assert float(med[g, m]) == statistics.median(vals)


def test_bootstrap_beyond_shared_memory_is_a_limit_error(gpu_ready):
    """256 metrics x groups of 128: the fold cannot fit one block; the call says so before launching."""
    from powermodeling_b200 import _native as N
    G, M, n = 1, 256, 128
    values = np.zeros((n, M))
    offsets = np.array([0, n], dtype=np.int32)
    seeds = np.array([1], dtype=np.uint64)
    out = [np.empty(G * M) for _ in range(3)]
    job = N.BootstrapJob(G, M, n, n, 1000, n, values.ctypes.data, offsets.ctypes.data, None, None,
                         seeds.ctypes.data, out[0].ctypes.data, out[1].ctypes.data, out[2].ctypes.data)
    assert N.library().pm_group_bootstrap(job) == -4     # PM_E_LIMIT
    assert "shared memory" in N.last_error()


@pytest.mark.parametrize("label,shape,seed", [("trapezoid", dict(points=2, repeats=4), 21),
                                               ("counter", dict(points=2, repeats=3, with_energy_counter=True), 22)])
def test_trials_csv_matches_reference(gpu_ready, tmp_path, label, shape, seed):
    """summarize on the GPU, written by write_summary: the metric columns of trials.csv equal the
    reference's file for the same records (tests/golden/summary_files.json.gz)."""
    import csv
    import io
    from powermodeling_b200.analysis import METRICS, summarize, write_summary
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    case = next(c for c in load_golden("summary_files.json.gz") if c["label"] == label)
    summary = summarize(make_sweep(SweepShape(**shape), seed), policy=ANALYSIS_POLICY)
    write_summary(summary, tmp_path)
    ours = list(csv.DictReader(io.StringIO((tmp_path / "trials.csv").read_text())))
    theirs = list(csv.DictReader(io.StringIO(case["files"]["trials.csv"])))
    assert [r["trial_id"] for r in ours] == [r["trial_id"] for r in theirs]
    exact = ("trial_id", "workload", "valid", "issues", "warnings", "energy_source", "count_energy_time_alignment_exact",
             "baseline_valid", "operational_idle_increment_eligible", "paired_active_reference_eligible",
             "board_power_w", "idle_power_w", "total_energy_j", "incremental_energy_j")
    numeric = tuple(METRICS) + ("duration_s", "power_limit_w")
    for mine, ref in zip(ours, theirs):
        for col in exact:
            assert mine[col] == ref[col], (mine["trial_id"], col, mine[col], ref[col])
        for col in numeric:
            a = float(mine[col]) if mine[col] else None
            b = float(ref[col]) if ref[col] else None
            assert close(a, b, rel=REL), (mine["trial_id"], col, a, b)


def _differences(want, got, path="") -> list[str]:
    """Paths at which two JSON values differ beyond the floating tolerance."""
    if isinstance(want, dict) and isinstance(got, dict):
        if want.keys() != got.keys():
            return [f"{path}: keys {sorted(want.keys() ^ got.keys())}"]
        return [d for k in want for d in _differences(want[k], got[k], f"{path}.{k}")]
    if isinstance(want, list) and isinstance(got, list):
        if len(want) != len(got):
            return [f"{path}: length {len(want)} != {len(got)}"]
        return [d for i, (a, b) in enumerate(zip(want, got)) for d in _differences(a, b, f"{path}[{i}]")]
    return [] if close(want, got, rel=REL) else [f"{path}: {want!r} != {got!r}"]


SELECTION_SECTIONS = ("within_clock_best", "cross_clock_best", "within_clock_best_total_energy",
                      "cross_clock_best_total_energy", "uncontrolled_clock_exploratory_best", "pareto_frontiers",
                      "active_control_associations", "verified_target_within_clock_best",
                      "verified_target_cross_clock_best", "verified_target_coverage", "empirical_gpu_energy_optima",
                      "empirical_gpu_overall_energy_optima", "exploratory_single_geometry_energy_optima",
                      "exploratory_single_geometry_overall_energy_optima", "metric_aliases", "notes")


def test_summary_selection_sections_match_reference(gpu_ready):
    """summarize's selection sections and evaluation over the GPU's groups equal the reference's
    summarize on the same records (the summary-file fixture: a trapezoid sweep and an energy-counter
    sweep)."""
    import json
    from powermodeling_b200.analysis import summarize
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    shapes = {"trapezoid": (SweepShape(points=2, repeats=4), 21),
              "counter": (SweepShape(points=2, repeats=3, with_energy_counter=True), 22)}
    for case in load_golden("summary_files.json.gz"):
        want = json.loads(case["files"]["summary.json"])
        shape, seed = shapes[case["label"]]
        got = json.loads(json.dumps(summarize(make_sweep(shape, seed), policy=ANALYSIS_POLICY)))
        assert want["within_clock_best"], case["label"]          # the fixture selects something
        for key in SELECTION_SECTIONS:
            assert got[key] == want[key], (case["label"], key)
        for key, value in want["selection_policy"].items():
            assert got["selection_policy"][key] == value, key
        # The evaluation reads trial-level values as well (1e-6 relative, as the trials themselves).
        assert not _differences(want["evaluation"], got["evaluation"]), (case["label"], _differences(want["evaluation"], got["evaluation"])[:5])
