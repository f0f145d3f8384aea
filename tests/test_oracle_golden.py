"""The oracle against the reference's own outputs (golden fixtures), on CPU."""
from __future__ import annotations

import pytest

from conftest import close, diff, load_golden
from oracle import analysis_oracle as O
from trial_builders import scenarios
from tests.golden.make_golden import records_digest

NUMERIC = ("duration_s", "total_energy_j", "board_power_w", "idle_power_w", "idle_energy_j", "incremental_energy_j",
           "incremental_power_w", "throughput_ops_s", "throughput_bytes_s", "counted_measure_operations",
           "counted_measure_logical_bytes", "count_energy_time_alignment_exact", "pj_per_op", "total_pj_per_op",
           "pj_per_logical_byte", "total_pj_per_flop", "operational_idle_increment_pj_per_flop",
           "total_pj_per_logical_bit", "operational_idle_increment_pj_per_logical_bit", "energy_source",
           "paired_active_reference_power_w", "paired_active_reference_energy_j", "active_reference_power_w",
           "active_reference_duration_s", "paired_active_reference_pj_per_flop",
           "paired_active_reference_pj_per_logical_bit", "throughput_elements_s", "throughput_rows_s",
           "counted_measure_elements", "row_width", "total_pj_per_element", "total_pj_per_row",
           "operational_idle_increment_pj_per_element", "operational_idle_increment_pj_per_row",
           "paired_active_reference_pj_per_element", "paired_active_reference_pj_per_row")
PHASE_NUMERIC = ("start_s", "end_s", "duration_s", "midpoint_s", "samples", "sample_interval_median_s",
                 "max_sample_gap_s", "integrated_power_energy_j", "power_w", "memory_rail_energy_j", "energy_counter_j",
                 "distinct_power_values", "observed_power_change_interval_median_s", "graphics_clock_mhz",
                 "temperature_c", "issues", "warnings")


@pytest.fixture(scope="module")
def golden():
    return {c["name"]: c for c in load_golden("analysis_trials.json.gz")["cases"]}


@pytest.mark.parametrize("name,record,policy", scenarios(), ids=[s[0] for s in scenarios()])
def test_oracle_matches_reference_trial(golden, name, record, policy):
    case = golden[name]
    assert case["digest"] == records_digest([record]), "scenario builder drifted from the fixture"
    got = O.analyze(record, policy)
    expected = case["expected"]
    problems = diff(expected, got, NUMERIC, rel=0.0)
    for phase, stats in expected["phases"].items():
        problems += [f"{phase}.{p}" for p in diff(stats, got["phases"].get(phase, {}), PHASE_NUMERIC, rel=0.0)]
    assert not problems, problems


def test_oracle_median_ci_matches_reference():
    data = load_golden("median_ci.json.gz")
    for case in data["cases"]:
        assert O.median_ci(case["values"], case["seed"]) == case["ci_1000"]
    for case in data["cases"][:12]:
        assert O.median_ci(case["values"], case["seed"], 10000) == case["ci_10000"]


def test_oracle_resample_stream_matches_reference():
    for s in load_golden("median_ci.json.gz")["streams"]:
        assert O.resample_indices(s["seed"], s["n"], len(s["rows"])) == s["rows"]


def test_oracle_sweep_numbers_match_reference():
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    for sweep in load_golden("analysis_sweeps.json.gz")["sweeps"]:
        records = make_sweep(SweepShape(**{k: tuple(v) if isinstance(v, list) else v for k, v in sweep["shape"].items()}), sweep["seed"])
        assert records_digest(records) == sweep["digest"]
        for record, expected in zip(records, sweep["trials"]):
            got = O.analyze(record, ANALYSIS_POLICY)
            assert not diff(expected, got, NUMERIC, rel=0.0)
