"""Generate the summary-file fixture from the reference implementation.

    python tests/golden/make_summary_golden.py <reference checkout>      (or PM_REFERENCE_TREE=<reference checkout>)

Runs the reference's summarize on two small synthetic sweeps, round-trips
each summary through JSON, and runs the reference's write_summary on it;
stores the text of summary.json, trials.csv, evaluation.json and
evaluation.csv (the summary is summary.json read back; the HTML view is not
kept) in tests/golden/summary_files.json.gz.
"""
from __future__ import annotations

import gzip
import json
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import analysis as ref  # the reference implementation
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    cases = []
    for label, shape, seed in (("trapezoid", SweepShape(points=2, repeats=4), 21),
                               ("counter", SweepShape(points=2, repeats=3, with_energy_counter=True), 22)):
        summary = ref.summarize(make_sweep(shape, seed), policy=ANALYSIS_POLICY)
        summary = json.loads(json.dumps(summary, allow_nan=False))
        with tempfile.TemporaryDirectory() as tmp:
            ref.write_summary(summary, tmp)
            files = {name: (Path(tmp) / name).read_text()
                     for name in ("summary.json", "trials.csv", "evaluation.json", "evaluation.csv")}
        cases.append({"label": label, "files": files})   # the summary itself is json.loads(summary.json)
    with gzip.open(HERE / "summary_files.json.gz", "wt") as f:
        json.dump(cases, f)
    print("wrote summary_files.json.gz", [len(c["files"]["trials.csv"]) for c in cases])


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit(f"usage: {Path(__file__).name} <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
