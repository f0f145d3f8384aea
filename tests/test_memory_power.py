"""Memory-rail sensor host logic against the reference (CPU): the per-sample checks and record assembly.

The window energies and phase midpoints the checks consume are the
reference's own (golden phase dictionaries), so this isolates
powermodeling_b200.memory_power from the GPU kernels; the GPU test checks the
whole path.
"""
from __future__ import annotations

import statistics

import pytest

from conftest import load_golden
from oracle import analysis_oracle as O
from powermodeling_b200 import memory_power as MP
from tests.golden.make_golden import records_digest
from trial_builders import memory_rail_group, memory_rail_scenarios

GOLDEN = load_golden("memory_power.json.gz")
CASES = {c["name"]: c for c in GOLDEN["cases"]}


@pytest.mark.parametrize("name,record", memory_rail_scenarios(), ids=[n for n, _ in memory_rail_scenarios()])
def test_trial_sensor_host_logic_matches_reference(name, record):
    case = CASES[name]
    assert case["digest"] == records_digest([record])
    expected = case["expected"]
    sensor = MP.trial_sensor(record, expected, expected["phases"], record["phases"], 2.5, 0.10)
    assert sensor == case["sensor"]


def test_group_sensor_host_logic_matches_reference():
    records = memory_rail_group()
    assert GOLDEN["group"]["digest"] == records_digest(records)
    trials = {t["trial_id"]: t for t in GOLDEN["group"]["trials"]}
    for g in GOLDEN["group"]["groups"]:
        observed = [trials[tid] for tid in g["trial_ids"]]
        valid = [t for t in observed if t["valid"]]
        for t in valid:
            t["hbm_memory_power"] = t["sensor"]
        cols = list(zip(*[MP.bootstrap_columns(t["sensor"]) for t in valid]))
        medians, intervals = [], []
        for column in cols:
            values = [v for v in column if v == v]
            medians.append(statistics.median(values) if values else None)
            intervals.append(O.median_ci(values, int(g["group_id"], 16), 1000))
        got = MP.group_sensor(valid, "hbm", observed, medians, intervals)
        assert got == g["sensor"]


def test_non_hbm_workloads_have_no_sensor():
    assert MP.trial_sensor({"workload": "l2"}, {}, {}, {}, 2.5, 0.1) is None
    assert MP.group_sensor([], "tensor", None, [], []) is None
