"""Generate the nonlinear count-contract fixture from the reference implementation.

    python tests/golden/make_nonlinear_golden.py <reference checkout>      (or PM_REFERENCE_TREE=<reference checkout>)

Runs the reference's powermodeling.nonlinear.count_issues (nonlinear.py:22-128)
on every record of tests/nonlinear_cases.cases() and writes the issue lists,
with a digest of each record, to tests/golden/nonlinear_contract.json.gz.
"""
from __future__ import annotations

import gzip
import hashlib
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import nonlinear_cases  # noqa: E402


def record_digest(record) -> str:
    return hashlib.sha256(json.dumps(record, sort_keys=True, default=repr).encode()).hexdigest()


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling.nonlinear import count_issues  # the reference implementation
    out = [{"name": name, "workload": workload, "digest": record_digest(record), "issues": count_issues(record, workload)}
           for name, workload, record in nonlinear_cases.cases()]
    with gzip.open(HERE / "nonlinear_contract.json.gz", "wt") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print(f"{len(out)} cases; {sum(1 for c in out if c['issues'])} with issues")


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit(f"usage: {Path(__file__).name} <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
