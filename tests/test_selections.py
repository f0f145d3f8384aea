"""Selections, energy optima, coverage, Pareto frontiers and control associations against the
reference's own functions on varied group sets (golden fixture, CPU)."""
from __future__ import annotations

import json

import pytest

from conftest import load_golden
from powermodeling_b200 import selections as S

CASES = load_golden("selections.json.gz")
FRACTION, MIN_REPEATS, NEAR = 0.95, 3, 0.05


def ours(groups: list) -> dict:
    out = {}
    for cross in (False, True):
        tag = "cross" if cross else "within"
        out[f"{tag}_best"] = S.best_conditions(groups, FRACTION, MIN_REPEATS, cross)
        out[f"{tag}_best_total"] = S.best_conditions(groups, FRACTION, MIN_REPEATS, cross, total_energy=True)
        out[f"{tag}_verified"] = S.best_conditions(groups, FRACTION, MIN_REPEATS, cross, True)
        out[f"{tag}_coverage"] = S.verification_coverage(groups, FRACTION, MIN_REPEATS, cross)
        out[f"{tag}_pareto"] = S.pareto_frontiers(groups, MIN_REPEATS, cross)
    out["exploratory"] = S.best_conditions(groups, FRACTION, MIN_REPEATS, True, exploratory_only=True)
    out["controls"] = S.control_associations(groups, MIN_REPEATS)
    for across in (False, True):
        for single in (False, True):
            out[f"optima_{int(across)}{int(single)}"] = S.energy_optima(
                groups, FRACTION, MIN_REPEATS, NEAR, 2, across_memory_domains=across, single_geometry_exploratory=single)
    return json.loads(json.dumps(out))


@pytest.mark.parametrize("memo", [False, True], ids=["direct", "memo"])
@pytest.mark.parametrize("case", CASES, ids=[str(c["seed"]) for c in CASES])
def test_sections_match_reference(case, memo):
    if memo:                      # the summary evaluates its sections with strata cached per group
        with S.stratum_memo():
            got = ours(case["groups"])
    else:
        got = ours(case["groups"])
    assert got.keys() == case["sections"].keys()
    for key, want in case["sections"].items():
        assert got[key] == want, key


def test_fixture_reaches_every_section():
    for key in CASES[0]["sections"]:
        assert any(c["sections"][key] for c in CASES), key


def test_read_geometry_flags_strides_offsets_and_slices():
    ok = S.read_geometry({"access": "read", "stride_elements": 1, "offset_bytes": 64, "threads": 256,
                          "working_set_bytes": 1 << 20}, "hbm")
    assert ok["status"] == "pass" and ok["energy_eligible"] and ok["requested_sector_efficiency_fraction"] == 1.0
    bad = S.read_geometry({"access": "read", "stride_elements": 2, "offset_bytes": 4, "threads": 100,
                           "working_set_bytes": 1 << 20}, "hbm")
    assert bad["status"] == "fail" and set(bad["reasons"]) == {
        "nonunit_word_stride", "offset_not_sector_aligned", "threads_not_complete_supported_warps"}
    l1 = S.read_geometry({"access": "read", "threads": 256, "working_set_bytes": 148 * 4096, "blocks": 148}, "l1")
    assert l1["effective_region_bytes"] == 4096 and l1["region_source"] == "floor(working_set_words/blocks)*4"
    assert S.read_geometry({"access": "copy"}, "hbm")["reasons"] == ["coalesced_read_energy_not_applicable"]


def test_summary_sections_from_the_references_groups():
    """The summary record's sections, computed here from the groups of the reference's own summaries
    (the summary-file fixture), equal the sections the reference wrote beside them."""
    from powermodeling_b200.analysis import AnalysisPolicy, summary_record
    from powermodeling_b200.synthetic import ANALYSIS_POLICY
    for case in load_golden("summary_files.json.gz"):
        want = json.loads(case["files"]["summary.json"])
        got = json.loads(json.dumps(summary_record(want["trials"], want["groups"], want["duplicate_trial_ids_ignored"],
                                                   0.95, 0.80, 3, 1000, AnalysisPolicy(**ANALYSIS_POLICY))))
        assert [k for k in got] == [k for k in want if k != "evaluation"]
        for key in got:
            assert got[key] == want[key], (case["label"], key)
