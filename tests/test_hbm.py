"""HBM bandwidth gate against the reference's own trial_bandwidth / group_bandwidth (golden fixture, CPU)."""
from __future__ import annotations

import json

import hbm_cases
from conftest import load_golden
from powermodeling_b200 import hbm

GOLDEN = load_golden("hbm_bandwidth.json.gz")


def _plain(obj):
    """The record as the fixture stores it (JSON, NaN and other non-JSON values as repr)."""
    return json.loads(json.dumps(obj, default=repr))


def test_trial_bandwidth_matches_reference():
    cases = hbm_cases.trial_cases()
    assert len(cases) == len(GOLDEN["trials"])
    got = [_plain(hbm.trial_bandwidth(r, t, s, f)) for r, t, s, f in cases]
    assert sum(1 for g in GOLDEN["trials"] if g and g["eligible"]) >= 100
    assert sum(1 for g in GOLDEN["trials"] if g and g["status"] == "fail") >= 100
    for i, (a, b) in enumerate(zip(got, GOLDEN["trials"])):
        assert a == b, i


def test_group_bandwidth_matches_reference():
    cases = hbm_cases.group_cases(hbm.trial_bandwidth)
    assert len(cases) == len(GOLDEN["groups"])
    for i, ((trials, workload, fraction), want) in enumerate(zip(cases, GOLDEN["groups"])):
        assert _plain(hbm.group_bandwidth(trials, workload, fraction)) == want, i
