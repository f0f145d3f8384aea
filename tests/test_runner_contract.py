"""This engine's powerbench records through the reference's own runner and count contracts (CPU).

The fixtures (tests/golden/make_runner_fixture.py): the reference's planner
built each trial's argv; this engine ran it on a B200 under its native
sampler; the reference's runner.capture_trial replayed the stored stdout and
samples, and its sfu/memory/nonlinear.count_issues checked the records.
"""
from __future__ import annotations

import json

import pytest

from conftest import ROOT, close, diff, load_golden
from powermodeling_b200 import contracts

PLAN = json.loads((ROOT / "tests" / "golden" / "runner_plan.json").read_text())
CAPTURES = {c["trial_id"]: c for c in load_golden("runner_captures.json.gz")}
CHECKS = {c["trial_id"]: c for c in load_golden("runner_checks.json.gz")}
TRIALS = {e["trial"]["trial_id"]: e["trial"] for e in PLAN}


def test_fixtures_cover_the_plan():
    assert set(CAPTURES) == set(CHECKS) == set(TRIALS)
    workloads = {t["workload"] for t in TRIALS.values()}
    assert {"hbm", "l1", "l2", "l2_latency", "tensor", "gemm", "control", "sfu_ex2", "softmax", "exp"} <= workloads
    assert sum(1 for t in TRIALS.values() if t.get("treatment_protocol")) >= 2


@pytest.mark.parametrize("trial_id", sorted(TRIALS))
def test_reference_runner_accepts_the_record(trial_id):
    check, trial = CHECKS[trial_id], TRIALS[trial_id]
    assert check["status"] == "complete" and check["runner_errors"] == [], check["runner_errors"]
    assert check["exclusivity_verified"] is True
    required = {"idle_pre", "measure", "idle_post"}
    if trial.get("treatment_protocol"):
        required |= {"active_reference", "warmup_reference", "warmup_treatment"}
    assert required <= set(check["phases"])
    assert CAPTURES[trial_id]["own_runner_errors"] == []


@pytest.mark.parametrize("trial_id", sorted(TRIALS))
def test_count_contracts_agree_with_the_references(trial_id):
    check, workload = CHECKS[trial_id], TRIALS[trial_id]["workload"]
    events = [json.loads(line) for line in CAPTURES[trial_id]["stdout"].splitlines()]
    bench = next(e for e in events if e["type"] == "result")
    reference = next((e for e in events if e["type"] == "active_reference_result"), None)
    assert check["sfu"] == check["memory"] == check["nonlinear"] == [] and check["sfu_reference"] == []
    assert contracts.sfu_count_issues(bench, workload) == check["sfu"]
    assert contracts.memory_count_issues(bench, workload) == check["memory"]
    assert contracts.nonlinear_count_issues(bench, workload) == check["nonlinear"]
    if reference is not None:
        assert contracts.sfu_count_issues(reference, workload, reference=True) == check["sfu_reference"]


@pytest.fixture(scope="module")
def runner_records():
    return load_golden("runner_records.json.gz")


@pytest.mark.gpu
def test_analysis_of_runner_records_matches_reference(gpu_ready, runner_records):
    """The reference runner's records of B200 telemetry, analysed here and by the reference."""
    from tests.golden.make_golden import PHASE_KEYS, TRIAL_KEYS
    from powermodeling_b200.analysis import analyze_trials
    from test_gpu_analysis import _differences
    got = analyze_trials(runner_records["records"])
    for expected, trial in zip(runner_records["trials"], got):
        problems = diff(expected, trial, TRIAL_KEYS)
        for phase, stats in expected["phases"].items():
            problems += [f"{phase}.{p}" for p in diff(stats, trial["phases"].get(phase, {}), PHASE_KEYS)]
        assert not problems, (expected["trial_id"], problems)
        # every field of the reference's trial dict, at the floating tolerance
        assert not _differences(expected, json.loads(json.dumps(trial))), (expected["trial_id"], _differences(expected, json.loads(json.dumps(trial)))[:6])
    assert any(t["valid"] for t in got) and any(t.get("paired_active_reference_power_w") for t in got)


@pytest.mark.gpu
def test_summary_of_runner_records_matches_reference(gpu_ready, runner_records):
    from powermodeling_b200.analysis import METRICS, summarize
    from test_gpu_analysis import _differences
    groups = summarize(runner_records["records"])["groups"]
    assert [g["group_id"] for g in groups] == [g["group_id"] for g in runner_records["groups"]]
    for got, expected in zip(groups, runner_records["groups"]):
        assert not _differences(expected, json.loads(json.dumps(got))), (expected["group_id"], _differences(expected, json.loads(json.dumps(got)))[:6])
    for got, expected in zip(groups, runner_records["groups"]):
        for metric in METRICS:
            assert close(expected.get(metric), got.get(metric)), (expected["group_id"], metric)
            assert close(expected["ci95"].get(metric), got["ci95"].get(metric)), (expected["group_id"], metric)
