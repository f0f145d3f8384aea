"""Generate the golden memory-rail sensor fixtures from the reference implementation.

    python tests/golden/make_memory_power_golden.py <reference checkout>      (or PM_REFERENCE_TREE=<reference checkout>)

Runs the reference's analyze_trial on tests/trial_builders.memory_rail_scenarios()
and its summarize on memory_rail_group(), keeping each trial's
``hbm_memory_power`` record and memory-rail aliases and each group's sensor
record, aliases and intervals.  Inputs are rebuilt by the tests and checked
by digest; tests/golden/memory_power.json.gz holds reference outputs only.
"""
from __future__ import annotations

import gzip
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from tests.golden.make_golden import pick, records_digest  # noqa: E402

ALIASES = ("memory_rail_power_w", "memory_rail_energy_j", "memory_rail_idle_power_w",
           "memory_rail_incremental_power_w", "memory_rail_incremental_energy_j")


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import analysis as ref
    from trial_builders import memory_rail_group, memory_rail_scenarios

    cases = []
    for name, record in memory_rail_scenarios():
        trial = ref.analyze_trial(record)
        cases.append({"name": name, "digest": records_digest([record]), "expected": pick(trial),
                      "sensor": trial.get("hbm_memory_power"), "aliases": {k: trial.get(k) for k in ALIASES}})
    records = memory_rail_group()
    summary = ref.summarize(records)
    groups = [{"group_id": g["group_id"], "trial_ids": g["trial_ids"], "valid_repeats": g["valid_repeats"],
               "sensor": g.get("hbm_memory_power"), "aliases": {k: g.get(k) for k in ALIASES},
               "alias_ci95": {k: g["ci95"].get(k) for k in ALIASES}} for g in summary["groups"]]
    trials = [{"trial_id": t["trial_id"], "valid": t["valid"], "sensor": t.get("hbm_memory_power")}
              for t in summary["trials"]]
    payload = {"cases": cases, "group": {"digest": records_digest(records), "groups": groups, "trials": trials}}
    with gzip.open(HERE / "memory_power.json.gz", "wt") as f:
        json.dump(payload, f, allow_nan=True, separators=(",", ":"))
    print("wrote memory_power.json.gz:", len(cases), "trials,", len(groups), "groups")


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit(f"usage: {Path(__file__).name} <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
