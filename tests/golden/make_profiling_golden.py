"""Generate the Nsight CSV reader fixture from the reference implementation.

    python tests/golden/make_profiling_golden.py <reference checkout>

(or PM_REFERENCE_TREE=<reference checkout>).  Runs the reference's
profiling.normalize_metric_value (profiling.py:91-130) on the cells of
tests/profiling_cases.py and its parse_ncu_csv (132-147) on the CSV texts
there, and writes the results to tests/golden/profiling.json.gz.
"""
from __future__ import annotations

import gzip
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import profiling  # the reference implementation
    from profiling_cases import CELLS, CSV_TEXTS
    cells = [[value, unit, list(profiling.normalize_metric_value(value, unit))] for value, unit in CELLS]
    texts = []
    for text in CSV_TEXTS:
        try:
            texts.append({"rows": profiling.parse_ncu_csv(text)})
        except ValueError as exc:
            texts.append({"error": str(exc)})
    with gzip.open(HERE / "profiling.json.gz", "wt") as f:
        json.dump({"cells": cells, "texts": texts, "metrics": list(profiling.METRICS)}, f)
    print(len(cells), "cells,", len(texts), "texts")


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit("usage: make_profiling_golden.py <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
