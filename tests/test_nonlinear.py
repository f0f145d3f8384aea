"""Streaming nonlinear workloads on the CPU: the count contract against the
reference's own count_issues (golden fixture) and the oracle's fill and
sampling rules."""
from __future__ import annotations

import numpy as np
import pytest

import nonlinear_cases
import workload_oracle as W
from conftest import load_golden
from golden.make_nonlinear_golden import record_digest
from oracle import nonlinear_oracle as O
from powermodeling_b200 import contracts

GOLDEN = load_golden("nonlinear_contract.json.gz")
CASES = nonlinear_cases.cases()


def test_fixture_covers_the_cases():
    assert [g["name"] for g in GOLDEN] == [name for name, _, _ in CASES]
    assert sum(1 for g in GOLDEN if not g["issues"]) >= 20          # consistent records are accepted
    assert sum(1 for g in GOLDEN if g["issues"]) >= 250             # and every planted mistake is caught


@pytest.mark.parametrize("index", range(len(CASES)), ids=[c[0] for c in CASES])
def test_count_issues_match_reference(index):
    name, workload, record = CASES[index]
    gold = GOLDEN[index]
    assert gold["digest"] == record_digest(record), "the case builder changed; regenerate the fixture"
    assert contracts.nonlinear_count_issues(record, workload) == gold["issues"], name
    assert O.count_issues(record, workload) == gold["issues"], name


def test_fill_is_exact_and_in_range():
    x = O.fill(1 << 16, seed=7)
    assert x.dtype == np.float32 and x.min() >= -4.0 and x.max() < 4.0
    assert np.all((x.astype(np.float64) * 8192.0) == np.round(x.astype(np.float64) * 8192.0))
    s = O.fill(4096, seed=7, shift=100.0)
    assert s.min() >= 96.0 and s.max() < 104.0
    g = O.fill(1024, seed=7 ^ 12345, gamma=True)
    assert g.min() >= 0.75 and g.max() < 1.25


def test_fill_words_agree_with_the_c_word_oracle():
    lib = W.lib()
    idx = np.array([0, 1, 2, 12345, 2 ** 33 + 17, 2 ** 63 + 5], dtype=np.uint64)
    assert [int(v) for v in O.random_words(idx)] == [lib.oracle_random_word(int(i)) for i in idx]


def test_sample_positions():
    assert O.sample_items(1) == [0]
    assert O.sample_items(3) == [0, 1, 2]
    assert O.sample_items(205) == [0, 29, 58, 87, 102, 145, 174, 204]
    assert len(set(O.sample_items(10 ** 6))) == 8


def test_reference_rule_accepts_double_results_and_rejects_a_planted_error():
    for function, width in (("exp", 0), ("tanh", 0), ("silu", 0), ("softmax", 129), ("rmsnorm", 129)):
        x, g = O.workload_inputs(function, 129 * 4, seed=3, width=width)
        e = O.expected(function, x, g, width)
        y = e.astype(np.float32)
        assert O.within_tolerance(y, e).all(), function
        bad = y.copy()
        bad[5] = bad[5] * np.float32(1.01) + np.float32(1e-3)
        assert not O.within_tolerance(bad, e)[5]
        if function == "softmax":
            assert O.softmax_rows_sum_to_one(y, width).all()
