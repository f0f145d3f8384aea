"""SFU and memory count contracts against the reference's own count_issues (golden fixture, CPU)."""
from __future__ import annotations

import pytest

import contract_cases
from conftest import load_golden
from golden.make_nonlinear_golden import record_digest
from powermodeling_b200 import contracts

GOLDEN = load_golden("count_contracts.json.gz")
SFU = contract_cases.sfu_cases()
MEMORY = contract_cases.memory_cases()


def test_fixture_covers_the_cases():
    assert [g["name"] for g in GOLDEN["sfu"]] == [c[0] for c in SFU]
    assert [g["name"] for g in GOLDEN["memory"]] == [c[0] for c in MEMORY]
    assert sum(1 for g in GOLDEN["sfu"] if not g["issues"]) >= 36       # every consistent record is accepted
    assert sum(1 for g in GOLDEN["sfu"] if g["issues"]) >= 500          # and the planted mistakes are caught
    assert sum(1 for g in GOLDEN["memory"] if g["issues"]) >= 50


@pytest.mark.parametrize("index", range(len(SFU)), ids=[c[0] for c in SFU])
def test_sfu_count_issues_match_reference(index):
    name, workload, reference, record = SFU[index]
    gold = GOLDEN["sfu"][index]
    assert gold["digest"] == record_digest(record), "the case builder changed; regenerate the fixture"
    assert contracts.sfu_count_issues(record, workload, reference=reference) == gold["issues"], name


@pytest.mark.parametrize("index", range(len(MEMORY)), ids=[c[0] for c in MEMORY])
def test_memory_count_issues_match_reference(index):
    name, workload, record = MEMORY[index]
    gold = GOLDEN["memory"][index]
    assert gold["digest"] == record_digest(record), "the case builder changed; regenerate the fixture"
    assert contracts.memory_count_issues(record, workload) == gold["issues"], name
