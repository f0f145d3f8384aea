"""Generate the full-trial fixture from the reference implementation.

    python tests/golden/make_trial_report_golden.py <reference checkout>

(or PM_REFERENCE_TREE=<reference checkout>).  Runs the reference's own
analyze_trial on every scenario record of tests/trial_builders.py and writes
its complete result dicts (every field, JSON round-tripped) with a digest of
each record to tests/golden/trial_reports.json.gz.  The records themselves
are rebuilt by the tests.  The runner-contract fixture holds the same for the
reference runner's records of B200 telemetry.
"""
from __future__ import annotations

import gzip
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE.parent))


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import analysis as ref  # the reference implementation
    from trial_builders import scenarios
    from tests.golden.make_golden import records_digest
    cases = []
    for name, record, policy in scenarios():
        result = json.loads(json.dumps(ref.analyze_trial(record, policy)))
        cases.append({"name": name, "digest": records_digest([record]), "expected": result})
    with gzip.open(HERE / "trial_reports.json.gz", "wt") as f:
        json.dump(cases, f)
    print(len(cases), "trials;", len({k for c in cases for k in c["expected"]}), "distinct keys")


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit("usage: make_trial_report_golden.py <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
