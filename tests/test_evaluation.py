"""The component evaluation against the reference's evaluate and its written files (CPU).

The fixture (tests/golden/make_evaluation_golden.py) holds the reference's
evaluation of summaries varied from its own summarize output, without a plan
and with complete, gapped, strict and role-refused plans; the planner's
policy check is the one piece taken as given (its error text is replayed).
"""
from __future__ import annotations

import json

import pytest

from conftest import load_golden
from powermodeling_b200 import evaluation as E
from powermodeling_b200.synthetic import SweepShape, make_sweep
from tests.golden.make_evaluation_golden import compact, digest, plateau_variant, vary_more

FIXTURE = load_golden("evaluation.json.gz")
BASE = FIXTURE["base"]
RECORDS = make_sweep(SweepShape(points=16, repeats=3), 31)


def _summary(seed: int) -> dict:
    groups, trials = vary_more(BASE["groups"], BASE["trials"], seed)
    if seed % 3 == 0:
        groups = plateau_variant(groups, seed)
    return dict(BASE, groups=groups, trials=trials)


def _validator(error):
    def check(plan):
        if error is not None:
            raise ValueError(error)
    return check


CASES = FIXTURE["cases"]


@pytest.mark.parametrize("case", CASES, ids=[f"{c['seed']}-{c['plan_kind']}" for c in CASES])
def test_evaluation_matches_reference(case, tmp_path):
    summary = _summary(case["seed"])
    got = E.evaluate(summary, plan=case["plan"], raw_records=RECORDS, plan_validator=_validator(case["plan_policy_error"]))
    got = json.loads(json.dumps(got))
    want = case["evaluation"]
    assert compact(got).keys() == want.keys()
    for key in want:
        if key != "components":
            assert compact(got)[key] == want[key], key
    assert len(got["components"]) == len(want["components"])
    for mine, theirs in zip(compact(got)["components"], want["components"]):
        for key in theirs:
            assert mine[key] == theirs[key], (theirs["stratum"]["workload"], key)
    paths = E.write_evaluation(got, tmp_path)
    files = {name: digest((tmp_path / name).read_text()) for name in case["file_digests"]}
    assert files == case["file_digests"]
    assert set(paths) == {"evaluation_json", "evaluation_csv"} | ({"hbm_memory_power_csv"} if "hbm-memory-power.csv" in files else set())


def test_fixture_reaches_the_evaluation_stages():
    evaluations = [c["evaluation"] for c in CASES]
    statuses = {r["status"] for e in evaluations for c in e["components"] for r in c["recommendations"]}
    assert {"diagnostic_only", "no_qualified_candidate", "provisional_candidate"} <= statuses
    assert {c["evaluation"]["coverage"]["status"] for c in CASES} >= {"complete", "incomplete", "unknown"}
    workloads = {c["stratum"]["workload"] for e in evaluations for c in e["components"]}
    assert {"hbm", "tensor", "gemm", "softmax", "sfu_ex2", "control", "l2_latency"} <= workloads
    assert any(c["input_scaling"]["curves"] for e in evaluations for c in e["components"])
    assert any(c["latency_points"] for e in evaluations for c in e["components"])
    assert any(r.get("factory_default_comparison", {}).get("status") == "available"
               for e in evaluations for c in e["components"] for r in c["recommendations"])


def test_policy_and_plan_errors():
    with pytest.raises(ValueError, match="minimum_resource_levels"):
        E.EvaluationPolicy(minimum_resource_levels=2)
    with pytest.raises(ValueError, match="fractions"):
        E.EvaluationPolicy(maximum_relative_ci_width=1.5)
    summary = _summary(0)
    with pytest.raises(ValueError, match="trials list"):
        E.evaluate(summary, plan={"trials": None})
    with pytest.raises(ValueError, match="Unsafe or missing trial_id"):
        E.evaluate(summary, plan={"trials": [{"trial_id": "../x", "workload": "tensor"}]})
    with pytest.raises(ValueError, match="Duplicate trial_id"):
        E.evaluate(summary, plan={"trials": [{"trial_id": "a", "workload": "tensor"}] * 2})
