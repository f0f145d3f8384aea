"""Generate the selections fixture from the reference implementation.

    python tests/golden/make_selections_golden.py <reference checkout>

(or PM_REFERENCE_TREE=<reference checkout>).  Builds group dicts with the
reference's own summarize on a synthetic sweep, then varies them (requested
clocks, launch geometries, workloads, verification and eligibility flags,
rates and energies, control groups) so every branch of the reference's
selection sections is reached, and runs its _selections,
_empirical_energy_optima, _verification_coverage, _pareto_frontiers and
_associate_controls (analysis.py:1104-1376) on each variant.  Writes the
groups and the sections to tests/golden/selections.json.gz.
"""
from __future__ import annotations

import copy
import gzip
import json
import os
import random
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

FRACTION, MIN_REPEATS, NEAR = 0.95, 3, 0.05
CLOCKS = ((1965, 3996), (1755, 3996), (1545, 3996), (1965, 2619), (1335, 2619))
GEOMETRIES = ({"blocks": 148, "threads": 128, "tensor_accumulators": 2}, {"blocks": 296, "threads": 256, "tensor_accumulators": 4},
              {"blocks": 592, "threads": 256, "tensor_accumulators": 1})


def vary(groups: list, seed: int) -> list:
    """A copy of ``groups`` with clocks, geometries, workloads, flags and values drawn from ``seed``."""
    rng = random.Random(seed)
    out = []
    for i, base in enumerate(groups):
        g = copy.deepcopy(base)
        gfx, mem = rng.choice(CLOCKS)
        g["config"]["graphics_clock_mhz"], g["config"]["memory_clock_mhz"] = gfx, mem
        g["graphics_clock_mhz"], g["memory_clock_mhz"] = gfx - rng.choice((0, 15)), mem
        g["config"].pop("point", None) if rng.random() < 0.3 else None
        g["resource_geometry"] = dict(rng.choice(GEOMETRIES))
        g["verified_selection_eligible"] = g["target_verified"] = rng.random() < 0.7
        g["operational_idle_increment_eligible"] = rng.random() < 0.85
        g["paired_active_reference_eligible"] = rng.random() < 0.6
        g["clock_comparison_controlled"] = rng.random() < 0.85
        g["valid_repeats"] = rng.choice((3, 3, 4, 2))
        scale = rng.uniform(0.6, 1.4)
        for key in ("pj_per_op", "total_pj_per_op", "total_pj_per_flop", "operational_idle_increment_pj_per_flop",
                    "paired_active_reference_pj_per_flop", "board_power_w"):
            if isinstance(g.get(key), (int, float)):
                g[key] *= scale
                if g["ci95"].get(key):
                    g["ci95"][key] = [v * scale for v in g["ci95"][key]]
        g["throughput_ops_s"] *= rng.uniform(0.9, 1.1)
        kind = rng.random()
        if kind < 0.15:                                     # an HBM read group
            g["workload"] = "hbm"
            g["config"].update(access="read", stride_elements=rng.choice((1, 1, 2)), offset_bytes=rng.choice((0, 0, 16)),
                               threads=256, working_set_bytes=1 << 30, read_cache_policy=rng.choice(("cg", "cg", "cs")))
            g["memory_coalescing_energy_eligible"] = rng.random() < 0.7
            g["throughput_bytes_s"] = rng.uniform(5e12, 7e12)
            for key in ("pj_per_logical_byte", "total_pj_per_logical_byte", "total_pj_per_logical_bit",
                        "operational_idle_increment_pj_per_logical_bit", "paired_active_reference_pj_per_logical_bit"):
                g[key] = rng.uniform(5, 40)
                g["ci95"][key] = [g[key] * 0.95, g[key] * 1.05]
            g["hbm_bandwidth"] = {"eligible": rng.random() < 0.7, "minimum_fraction": 0.8}
        elif kind < 0.25:                                   # an SFU group with its paired delta
            g["workload"] = "sfu_ex2"
            g["throughput_sfu_instructions_s"] = rng.uniform(3e12, 4.5e12)
            g["sfu_reference_delta_pj_per_instruction"] = g["paired_active_reference_pj_per_instruction"] = rng.uniform(0.5, 3)
            g["ci95"]["sfu_reference_delta_pj_per_instruction"] = [0.4, 3.2]
            g["sfu_reference_delta_positive_optimum_eligible"] = rng.random() < 0.8
        elif kind < 0.32:                                   # an active-control group
            g["workload"] = "control"
        elif kind < 0.36:
            g["experiment_role"] = "diagnostic_probe"
        g["group_id"] = f"{seed:02d}{i:014x}"
        out.append(g)
    return out


def sections(ref, groups: list) -> dict:
    out = {}
    for cross in (False, True):
        tag = "cross" if cross else "within"
        out[f"{tag}_best"] = ref._selections(groups, FRACTION, MIN_REPEATS, cross)
        out[f"{tag}_best_total"] = ref._selections(groups, FRACTION, MIN_REPEATS, cross, total_energy=True)
        out[f"{tag}_verified"] = ref._selections(groups, FRACTION, MIN_REPEATS, cross, True)
        out[f"{tag}_coverage"] = ref._verification_coverage(groups, FRACTION, MIN_REPEATS, cross)
        out[f"{tag}_pareto"] = ref._pareto_frontiers(groups, MIN_REPEATS, cross)
    out["exploratory"] = ref._selections(groups, FRACTION, MIN_REPEATS, True, exploratory_only=True)
    out["controls"] = ref._associate_controls(groups, MIN_REPEATS)
    for across in (False, True):
        for single in (False, True):
            out[f"optima_{int(across)}{int(single)}"] = ref._empirical_energy_optima(
                groups, FRACTION, MIN_REPEATS, NEAR, 2, across_memory_domains=across, single_geometry_exploratory=single)
    return out


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import analysis as ref  # the reference implementation
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    summary = ref.summarize(make_sweep(SweepShape(points=24, repeats=3), 31), policy=ANALYSIS_POLICY)
    groups = json.loads(json.dumps(summary["groups"], allow_nan=False))
    cases = [{"seed": seed, "groups": vary(groups, seed)} for seed in range(12)]
    for case in cases:
        case["sections"] = json.loads(json.dumps(sections(ref, case["groups"])))
    with gzip.open(HERE / "selections.json.gz", "wt") as f:
        json.dump(cases, f)
    nonempty = {k: sum(bool(c["sections"][k]) for c in cases) for k in cases[0]["sections"]}
    print(len(cases), "cases; non-empty sections per key:", nonempty)


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit("usage: make_selections_golden.py <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
