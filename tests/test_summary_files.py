"""write_summary: summary.json and trials.csv equal to the reference's files for the same summary."""
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
    assert set(paths) == {"summary_json", "trials_csv"}
    for name in ("summary.json", "trials.csv"):
        assert (tmp_path / "out" / name).read_text() == case["files"][name], name


def test_non_finite_numbers_are_refused(tmp_path):
    with pytest.raises(ValueError):
        write_summary({"trials": [], "groups": [{"board_power_w": float("nan")}]}, tmp_path)
