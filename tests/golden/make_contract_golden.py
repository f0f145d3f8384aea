"""Generate the SFU and memory count-contract fixture from the reference implementation.

    python tests/golden/make_contract_golden.py <reference checkout>

(or PM_REFERENCE_TREE=<reference checkout>).  Runs the reference's
powermodeling.sfu.count_issues (sfu.py:23-115) and
powermodeling.memory.count_issues (memory.py:114-144) on every record of
tests/contract_cases and writes the issue lists, with a digest of each
record, to tests/golden/count_contracts.json.gz.
"""
from __future__ import annotations

import gzip
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import contract_cases  # noqa: E402
from golden.make_nonlinear_golden import record_digest  # noqa: E402


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import memory, sfu  # the reference implementation
    out = {"sfu": [{"name": name, "workload": workload, "reference": reference_arm, "digest": record_digest(record),
                    "issues": sfu.count_issues(record, workload, reference=reference_arm)}
                   for name, workload, reference_arm, record in contract_cases.sfu_cases()],
           "memory": [{"name": name, "workload": workload, "digest": record_digest(record),
                       "issues": memory.count_issues(record, workload)}
                      for name, workload, record in contract_cases.memory_cases()]}
    with gzip.open(HERE / "count_contracts.json.gz", "wt") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    for kind, rows in out.items():
        print(f"{kind}: {len(rows)} cases; {sum(1 for c in rows if c['issues'])} with issues")


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit("usage: make_contract_golden.py <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
