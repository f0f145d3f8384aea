"""write_summary: summary.json, trials.csv and the evaluation files equal to the reference's for the same summary."""
from __future__ import annotations

import json

import pytest

from conftest import load_golden
from powermodeling_b200.analysis import write_summary

CASES = load_golden("summary_files.json.gz")


@pytest.mark.parametrize("case", CASES, ids=[c["label"] for c in CASES])
def test_files_equal_the_references(case, tmp_path):
    summary = json.loads(case["files"]["summary.json"])
    paths = write_summary(summary, tmp_path / "out")
    assert set(paths) == {"summary_json", "trials_csv", "evaluation_json", "evaluation_csv"}
    for name in ("summary.json", "trials.csv", "evaluation.json", "evaluation.csv"):
        assert (tmp_path / "out" / name).read_text() == case["files"][name], name


def test_non_finite_numbers_are_refused(tmp_path):
    with pytest.raises(ValueError):
        write_summary({"trials": [], "groups": [{"board_power_w": float("nan")}]}, tmp_path)


@pytest.mark.parametrize("case", CASES, ids=[c["label"] for c in CASES])
def test_evaluation_of_the_references_summary(case):
    """evaluate() over the reference's own summary equals the evaluation that summary carries."""
    from powermodeling_b200.evaluation import evaluate
    from powermodeling_b200.synthetic import SweepShape, make_sweep
    shapes = {"trapezoid": (SweepShape(points=2, repeats=4), 21),
              "counter": (SweepShape(points=2, repeats=3, with_energy_counter=True), 22)}
    summary = json.loads(case["files"]["summary.json"])
    want = summary.pop("evaluation")
    shape, seed = shapes[case["label"]]
    assert json.loads(json.dumps(evaluate(summary, raw_records=make_sweep(shape, seed)))) == want
