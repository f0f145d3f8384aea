"""Memory-rail sensor records through the GPU analysis, against the reference's outputs."""
from __future__ import annotations

import pytest

from conftest import load_golden
from tests.golden.make_golden import records_digest
from trial_builders import memory_rail_group, memory_rail_scenarios

pytestmark = pytest.mark.gpu
GOLDEN = load_golden("memory_power.json.gz")
CASES = {c["name"]: c for c in GOLDEN["cases"]}


@pytest.mark.parametrize("name,record", memory_rail_scenarios(), ids=[n for n, _ in memory_rail_scenarios()])
def test_trial_sensor_matches_reference(gpu_ready, name, record):
    from powermodeling_b200.analysis import analyze_trial
    case = CASES[name]
    assert case["digest"] == records_digest([record])
    got = analyze_trial(record)
    assert got["hbm_memory_power"] == case["sensor"]
    for alias, value in case["aliases"].items():
        assert got.get(alias) == value, (alias, value, got.get(alias))


def test_group_sensor_matches_reference(gpu_ready):
    from powermodeling_b200.analysis import summarize
    records = memory_rail_group()
    assert GOLDEN["group"]["digest"] == records_digest(records)
    summary = summarize(records)
    assert len(summary["groups"]) == len(GOLDEN["group"]["groups"])
    for got, exp in zip(summary["groups"], GOLDEN["group"]["groups"]):
        assert got["group_id"] == exp["group_id"]
        assert got["hbm_memory_power"] == exp["sensor"]
        for alias, value in exp["aliases"].items():
            assert got.get(alias) == value, alias
            assert got["ci95"].get(alias) == exp["alias_ci95"][alias], alias
