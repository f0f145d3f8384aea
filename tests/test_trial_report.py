"""The reporting fields of a trial record against the reference's analyze_trial (CPU).

complete_trial() receives the reference's own numeric result with every
reporting field removed and must restore each one as the reference wrote it.
The measure window's samples (validation_binding) and the memory-rail sources
need the packed samples and are compared on the GPU, where the whole trial
dict is checked (tests/test_runner_contract.py)."""
from __future__ import annotations

import copy
import json

import pytest

from conftest import close, load_golden
from trial_builders import scenarios
from powermodeling_b200.analysis import AnalysisPolicy
from powermodeling_b200.trial_report import complete_trial
from tests.golden.make_golden import records_digest

REPORT_KEYS = ("memory_access_geometry", "memory_coalescing", "memory_coalescing_energy_eligible", "target_verified",
               "validation", "profile_rates_summary", "profiler_suitability_status", "ncu_status", "ncu_assessment",
               "ncu_target_suitability", "ncu_utilization_status", "verified_selection_eligible",
               "dynamic_attribution_eligible", "diagnostic_only", "physical_traffic_energy", "latency_probe",
               "kernel_resources", "execution_diagnostics", "memory_accesses_per_thread_iteration", "operation_unit",
               "numerical_validation", "model_features", "feature_units", "feature_provenance", "power_provenance",
               "power_scope", "power_usage_semantics", "treatment_outcome_kind", "idle_baseline_estimator",
               "idle_increment_interpretation", "baseline_kind", "baseline_power_scope", "dynamic_attribution_note",
               "attribution", "throughput_timebase", "paired_active_reference_interpretation",
               "element_count_convention", "row_operation_convention", "latency_diagnostics",
               "control_subtraction_note", "sfu_reference_delta_positive_optimum_eligible",
               "sfu_instruction_count_convention", "sfu_reference_delta_estimator", "sfu_hardware_attribution_proven",
               "sfu_reference_delta_diagnostics", "energy_peak_population_eligible", "measurement_diagnostics")
ON_GPU_ONLY = ("validation_binding", "memory_rail_sources")


def _cases():
    golden = {c["name"]: c for c in load_golden("trial_reports.json.gz")}
    out = []
    for name, record, policy in scenarios():
        case = golden[name]
        assert case["digest"] == records_digest([record])
        out.append((name, record, policy, case["expected"]))
    runner = load_golden("runner_records.json.gz")
    for record, expected in zip(runner["records"], runner["trials"]):
        out.append(("runner-" + record["trial_id"], record, None, expected))
    return out


CASES = _cases()


@pytest.mark.parametrize("name,record,policy,expected", CASES, ids=[c[0] for c in CASES])
def test_reporting_fields_match_reference(name, record, policy, expected):
    numeric = {k: copy.deepcopy(v) for k, v in expected.items() if k not in REPORT_KEYS + ON_GPU_ONLY}
    trim_s = AnalysisPolicy(**(policy or {})).trim_s
    got = complete_trial(record, numeric, trim_s, [], [])
    for key in REPORT_KEYS:
        assert (key in got) == (key in expected), key
        if key in expected:
            assert close(expected[key], got[key]), (key, expected[key], got[key])


def test_every_reference_field_is_covered():
    keys = {k for _, _, _, expected in CASES for k in expected}
    from powermodeling_b200 import analysis
    import inspect
    import re
    source = inspect.getsource(analysis)
    numeric = {k for k in keys if re.search(rf'"{k}"\s*:|\b{k}=|\["{k}"\]\s*=', source)}
    assert keys - numeric - set(REPORT_KEYS) - set(ON_GPU_ONLY) == set()


GROUP_REPORT_KEYS = ("memory_access_geometry", "memory_coalescing", "memory_coalescing_energy_eligible",
                     "kernel_resources", "execution_diagnostics", "memory_accesses_per_thread_iteration",
                     "target_verified", "verified_selection_eligible", "ncu_status", "sfu_reference_delta_measurement_valid",
                     "sfu_reference_delta_ci_crosses_zero", "sfu_reference_delta_positive_optimum_eligible",
                     "sfu_hardware_attribution_proven", "sfu_reference_delta_estimator", "sfu_reference_delta_issues",
                     "sfu_reference_delta_uncertainty", "ncu_target_suitability", "ncu_utilization_status",
                     "measurement_diagnostics", "energy_peak_population_eligible", "sfu_reference_delta_diagnostics")


def _summaries():
    import json
    out = []
    for case in load_golden("summary_files.json.gz"):
        summary = json.loads(case["files"]["summary.json"])
        out.append((case["label"], summary["trials"], summary["groups"]))
    runner = load_golden("runner_records.json.gz")
    out.append(("runner", runner["trials"], runner["groups"]))
    return out


@pytest.mark.parametrize("label,trials,groups", _summaries(), ids=lambda v: v if isinstance(v, str) else "")
def test_group_reporting_fields_match_reference(label, trials, groups):
    from powermodeling_b200.trial_report import complete_group
    by_id = {t["trial_id"]: t for t in trials}
    for group in groups:
        members = [by_id[i] for i in group["trial_ids"]]
        valid, seen = [], set()
        for t in members:
            if not t["valid"] or (t.get("repeat_index") is not None and t["repeat_index"] in seen):
                continue
            seen.add(t.get("repeat_index"))
            valid.append(t)
        stripped = {k: copy.deepcopy(v) for k, v in group.items() if k not in GROUP_REPORT_KEYS}
        stripped["ci95"].pop("paired_active_reference_pj_per_instruction", None) if group["workload"].startswith("sfu") else None
        if group["workload"].startswith("sfu"):
            stripped["ci95"]["paired_active_reference_pj_per_instruction"] = None
        got = complete_group(stripped, members[0], valid, 3)
        for key in GROUP_REPORT_KEYS:
            assert (key in got) == (key in group), (label, key)
            if key in group:
                assert close(group[key], got[key]), (label, group["workload"], key, group[key], got[key])
        assert close(group["ci95"], got["ci95"]), (label, "ci95")


def test_native_binding_samples_equal_the_python_statement():
    from powermodeling_b200 import _packnative
    from powermodeling_b200.trial_report import binding_samples

    class Sample(dict):
        def get(self, key, default=None):
            return "own"
    samples = [{"graphics_clock_mhz": 1965, "memory_clock_mhz": 3996}, {"graphics_clock_mhz": 1965, "memory_clock_mhz": 3996},
               {"graphics_clock_mhz": 1965.0, "memory_clock_mhz": 3996}, {"graphics_clock_mhz": True, "memory_clock_mhz": 3996},
               {"graphics_clock_mhz": 1, "memory_clock_mhz": 3996}, {"graphics_clock_mhz": float("nan")},
               {"graphics_clock_mhz": float("nan")}, {"graphics_clock_mhz": 1.5}, {}, {},
               Sample(graphics_clock_mhz=1), {"memory_clock_mhz": None, "t_s": 2.0}]
    n = len(samples)
    for lo, hi in ((0, n), (1, 3), (4, 4), (-2, n + 4), (2, 7)):
        want = binding_samples(samples[max(lo, 0):min(hi, n)])
        got = _packnative.binding_samples(samples, lo, hi)
        assert json.dumps(got) == json.dumps(want) and len(got) == len(want)
    shared = _packnative.binding_samples(samples, 0, 2)
    assert shared[0] is shared[1]                   # equal clocks: one entry object
    with pytest.raises(AttributeError):
        _packnative.binding_samples([3], 0, 1)
