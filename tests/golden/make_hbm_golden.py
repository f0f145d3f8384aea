"""Generate the HBM bandwidth-gate fixture from the reference implementation.

    python tests/golden/make_hbm_golden.py <reference checkout>

(or PM_REFERENCE_TREE=<reference checkout>).  Runs the reference's
powermodeling.hbm_bandwidth.trial_bandwidth and group_bandwidth
(hbm_bandwidth.py:42-125) on tests/hbm_cases and writes their records to
tests/golden/hbm_bandwidth.json.gz (NaN written as the string "nan").
"""
from __future__ import annotations

import gzip
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import hbm_cases  # noqa: E402


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import hbm_bandwidth as H  # the reference implementation
    trials = [H.trial_bandwidth(r, t, s, f) for r, t, s, f in hbm_cases.trial_cases()]
    groups = [H.group_bandwidth(ts, w, f) for ts, w, f in hbm_cases.group_cases(H.trial_bandwidth)]
    with gzip.open(HERE / "hbm_bandwidth.json.gz", "wt") as f:
        json.dump({"trials": trials, "groups": groups}, f, indent=0, default=repr)
    print(f"{len(trials)} trials ({sum(bool(t and t['eligible']) for t in trials)} eligible), {len(groups)} groups")


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit("usage: make_hbm_golden.py <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
