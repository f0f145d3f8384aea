"""Generate the evaluation fixture from the reference implementation.

    python tests/golden/make_evaluation_golden.py <reference checkout>

(or PM_REFERENCE_TREE=<reference checkout>).  Builds summaries from the
reference's own summarize on synthetic sweeps, then varies their groups and
trials so every stage of the reference's evaluate (evaluation.py:436-640) is
reached: workloads of every family (HBM, Tensor, GEMM, SFU and complete
functions on auto-grid input-size curves, control, latency), clocks with the
advertised-default and 1110 MHz anchors, geometries, profiler status,
intervals of every width, profiler checks, latency probes and sampled checks.
Runs the reference's evaluate on each (without a plan, and with plans that are
complete, incomplete, mismatched or refused by the planner's policy) and its
dashboard.write_evaluation, keeping the evaluation (each representative
trace's points as a digest), digests of the written files and the policy
error each plan raised, in tests/golden/evaluation.json.gz.
"""
from __future__ import annotations

import copy
import gzip
import json
import os
import random
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden.make_selections_golden import vary  # noqa: E402

CURVE_Q = (1 << 20, 1 << 22, 1 << 24, 1 << 26)
NCU = ("pass", "pass", "fail", "unprofiled", "inconclusive")


def _ci(rng, value, width):
    return [value * (1 - width / 2), value * (1 + width / 2)]


def vary_more(groups: list, trials: list, seed: int) -> tuple[list, list]:
    """Evaluation-specific variation on top of the selections fixture's."""
    rng = random.Random(1000 + seed)
    groups = vary(groups, seed)
    trials = copy.deepcopy(trials)
    by_id = {t["trial_id"]: t for t in trials}
    curve_base = None
    for i, g in enumerate(groups):
        g["ncu_status"] = rng.choice(NCU)
        g["target_verified"] = g["ncu_status"] == "pass" and rng.random() < 0.9
        g["count_energy_time_alignment_exact"] = rng.random() < 0.9
        g["repeats"] = g["valid_repeats"] + rng.choice((0, 0, 1))
        cfg = g["config"]
        if rng.random() < 0.2:
            cfg["clock_selection_reasons"] = ["advertised_default_fixed_pair"]
        if rng.random() < 0.15:
            cfg["graphics_clock_mhz"] = 1110
        # interval widths around the 10 % gate
        for key in list(g["ci95"]):
            value = g.get(key)
            if isinstance(value, (int, float)) and not isinstance(value, bool) and value and g["ci95"][key]:
                g["ci95"][key] = _ci(rng, value, rng.choice((0.02, 0.05, 0.08, 0.15)))
        kind = rng.random()
        if g["workload"] == "tensor" and kind < 0.25:                  # a softmax input-size curve
            g["workload"] = "softmax"
            q = CURVE_Q[i % len(CURVE_Q)]
            contract = {"row_width": 1024, "working_set_bytes": q * 4, "input_elements": q, "grid_mode": "auto",
                        "input_precision": "fp32", "math_implementation": "cuda_fp32_q_grid_v2",
                        "kernel_implementation_version": "nl_v2", "block_completion_count_source": "device",
                        "rms_epsilon": None, "affine_gamma": None, "nonlinear_input_distribution": "uniform"}
            curve_base = curve_base or {k: cfg.get(k) for k in ("graphics_clock_mhz", "memory_clock_mhz")}
            cfg.update(curve_base)
            g["nonlinear_contract"] = contract
            g["experiment_contract"] = {k: v for k, v in contract.items()}
            g["resource_geometry"] = {"blocks": q // 1024, "threads": 256}
            g["throughput_elements_s"] = rng.uniform(5e11, 6e11)
            g["ci95"]["throughput_elements_s"] = _ci(rng, g["throughput_elements_s"], 0.04)
            for prefix in ("total_", "operational_idle_increment_", "paired_active_reference_"):
                g[prefix + "pj_per_element"] = rng.uniform(20, 40)
                g["ci95"][prefix + "pj_per_element"] = _ci(rng, g[prefix + "pj_per_element"], 0.05)
                g[prefix + "pj_per_row"] = g[prefix + "pj_per_element"] * 1024
            g["verified_selection_eligible"] = True
        elif g["workload"] == "tensor" and kind < 0.32:
            g["workload"] = "gemm"
            n = rng.choice((2048, 4096, 8192))
            g["resource_geometry"] = {"gemm_m": n, "gemm_n": n, "gemm_k": n}
        elif g["workload"] == "tensor" and kind < 0.36:
            g["workload"] = "l2_latency"
        elif g["workload"] == "sfu_ex2" and rng.random() < 0.6:
            lanes = rng.choice((148 * 256, 296 * 256, 592 * 256))
            g["sfu_contract"] = {"sfu_lanes": lanes, "sfu_chains": 4, "grid_mode": "auto",
                                 "math_implementation": "ptx_approx_register_v1", "block_completion_count_source": "device"}
            g["sfu_reference_delta_measurement_valid"] = rng.random() < 0.8
        for t_id in g["trial_ids"]:
            t = by_id.get(t_id)
            if t is None:
                continue
            if rng.random() < 0.3:
                t["ncu_assessment"] = {"checks": [{"name": "target_kernel", "status": rng.choice(("pass", "fail"))},
                                                  {"name": "dram_bytes", "status": "pass"}],
                                       "traffic_amplification": rng.choice((None, 1.02, 1.4))}
            if rng.random() < 0.2:
                t["numerical_validation"] = {"status": "pass", "samples": 16}
            if rng.random() < 0.2:
                t["profile_rates_summary"] = {"dram_gbs": rng.uniform(1000, 7000)}
            if g["workload"] == "l2_latency":
                t["latency_probe"] = {"per_sm": {str(s): {"cycles_per_access": rng.choice((0, 290.5, 310.0))}
                                                 for s in range(3)}}
            if rng.random() < 0.1:
                t["valid"] = False
                t["issues"] = ["active_throttling"]
    return groups, trials


QUALIFIED = {"target_verified": True, "ncu_status": "pass", "verified_selection_eligible": True,
             "count_energy_time_alignment_exact": True, "clock_comparison_controlled": True, "valid_repeats": 3,
             "repeats": 3, "operational_idle_increment_eligible": True, "paired_active_reference_eligible": True,
             "experiment_role": "energy_characterization"}


def _qualify(g: dict, rng, rate: str, rate_value: float) -> None:
    g.update(QUALIFIED)
    g[rate] = rate_value
    g["ci95"][rate] = _ci(rng, rate_value, 0.02)
    for key, value in list(g.items()):
        if "_pj_per_" in key or key.startswith("total_pj") or key.startswith("pj_per"):
            if isinstance(value, (int, float)) and not isinstance(value, bool):
                g[key] = abs(value) or 1.0
                g["ci95"][key] = _ci(rng, g[key], 0.04)


def plateau_variant(groups: list, seed: int) -> list:
    """Qualified groups for the later stages: four Tensor groups at one clock pair and three
    resource levels with rates within 1 % (a resource plateau), matched anchor copies of them at
    the advertised default pair and at 1110 MHz, and the softmax curve made qualified near its
    peak (an input-size plateau)."""
    rng = random.Random(7000 + seed)
    tensor = [g for g in groups if g["workload"] == "tensor"][:4]
    geometries = ({"blocks": 148, "threads": 128, "tensor_accumulators": 2}, {"blocks": 296, "threads": 256, "tensor_accumulators": 4},
                  {"blocks": 592, "threads": 256, "tensor_accumulators": 1}, {"blocks": 1184, "threads": 256, "tensor_accumulators": 1})
    anchors = []
    for g, geometry in zip(tensor, geometries):
        g["config"].update(graphics_clock_mhz=1965, memory_clock_mhz=3996, clock_selection_reasons=[])
        g["resource_geometry"] = dict(geometry)
        _qualify(g, rng, "throughput_ops_s", 2.0e15 * rng.uniform(0.99, 1.0))
        for tag, gfx in (("advertised_default_fixed_pair", 1800), (None, 1110)):
            twin = copy.deepcopy(g)
            twin["group_id"] = g["group_id"][:-2] + ("ad" if tag else "11")
            twin["config"].update(graphics_clock_mhz=gfx, clock_selection_reasons=[tag] if tag else [])
            for key, value in list(twin.items()):
                if "pj_" in key and isinstance(value, float):
                    twin[key] = value * rng.uniform(1.02, 1.3)
                    twin["ci95"][key] = _ci(rng, twin[key], 0.03)
            anchors.append(twin)
    for g in [g for g in groups if g["workload"] == "softmax"]:
        _qualify(g, rng, "throughput_elements_s", 6.0e11 * rng.uniform(0.985, 1.0))
        twin = copy.deepcopy(g)            # a second geometry at the same Q (and a second curve)
        twin["group_id"] = g["group_id"][:-2] + "t1"
        twin["resource_geometry"]["threads"] = 128
        _qualify(twin, rng, "throughput_elements_s", 6.0e11 * rng.uniform(0.985, 1.0))
        anchors.append(twin)
    return groups + anchors


def digest(value) -> str:
    import hashlib
    text = value if isinstance(value, str) else json.dumps(value, sort_keys=True)
    return hashlib.sha256(text.encode()).hexdigest()


def compact(evaluation: dict) -> dict:
    """The evaluation with each representative trace's points replaced by their count and digest."""
    out = copy.deepcopy(evaluation)
    for comp in out["components"]:
        example = comp.get("measurement_example")
        if example:
            points = example.pop("points")
            example["points_digest"] = {"count": len(points), "sha256": digest(points), "head": points[:2]}
    return out


def plan_for(summary: dict, seed: int, kind: str) -> dict:
    """A plan over the summary's trials: complete, with missing/mismatched/unexpected trials, or strict."""
    rng = random.Random(5000 + seed)
    rows = []
    for t in summary["trials"]:
        cfg = t.get("config") or {}
        row = {"trial_id": t["trial_id"], "condition_id": t.get("condition_id"), "workload": t["workload"],
               "repeat": t.get("repeat_index"),
               "clocks": {"graphics_mhz": cfg.get("graphics_clock_mhz"), "memory_mhz": cfg.get("memory_clock_mhz")},
               "parameters": {}}
        if t.get("experiment_role", "legacy_unspecified") != "legacy_unspecified":
            row["experiment_role"] = t["experiment_role"]
        rows.append(row)
    plan = {"trials": rows, "study_design": "diagnostic", "device": {}}
    if kind == "gaps":
        del rows[rng.randrange(len(rows))]                        # an unexpected trial
        rows.append(dict(rows[0], trial_id="never-ran-0"))         # a missing trial
        rows[1]["clocks"] = {"graphics_mhz": 1, "memory_mhz": 2}   # a mismatched trial
        rows[2]["treatment_protocol"] = {"order": "AB"}
    elif kind == "strict":
        plan["study_design"] = "energy_sweep"
        plan["clock_sweep_coverage"] = {"advertised_default": {"status": "included", "graphics_mhz": 1965,
                                                                "memory_mhz": 3996}}
    elif kind == "bad_role":
        rows[0]["experiment_role"] = None
    return plan


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import analysis as ref  # the reference implementation
    from powermodeling import evaluation as ref_eval
    from powermodeling.dashboard import write_evaluation
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(points=16, repeats=3), 31)
    base = json.loads(json.dumps(ref.summarize(records, policy=ANALYSIS_POLICY), allow_nan=False))
    base.pop("evaluation")
    cases = []
    for seed in range(8):
        groups, trials = vary_more(base["groups"], base["trials"], seed)
        if seed % 3 == 0:
            groups = plateau_variant(groups, seed)
        summary = dict(base, groups=groups, trials=trials)
        for kind in ("none", "complete", "gaps", "strict", "bad_role") if seed < 3 else ("none",):
            plan = None if kind == "none" else plan_for(summary, seed, kind)
            try:
                evaluation = json.loads(json.dumps(ref_eval.evaluate(summary, plan=plan, raw_records=records)))
            except ValueError as exc:                              # the plan was refused outright
                cases.append({"seed": seed, "plan_kind": kind, "plan": plan, "raises": str(exc)})
                continue
            with tempfile.TemporaryDirectory() as tmp:
                paths = write_evaluation(evaluation, tmp)
                files = {Path(p).name: digest(Path(p).read_text()) for k, p in paths.items() if not p.endswith(".html")}
            cases.append({"seed": seed, "plan_kind": kind, "plan": plan, "evaluation": compact(evaluation),
                          "file_digests": files, "plan_policy_error": evaluation["coverage"].get("plan_policy_error")})
    with gzip.open(HERE / "evaluation.json.gz", "wt") as f:
        json.dump({"base": base, "cases": cases}, f)
    reached = {"recommendation statuses": sorted({r["status"] for c in cases if "evaluation" in c
                                                  for comp in c["evaluation"]["components"] for r in comp["recommendations"]}),
               "workloads": sorted({comp["stratum"]["workload"] for c in cases if "evaluation" in c
                                    for comp in c["evaluation"]["components"]}),
               "plateaus": sorted({r.get("saturation_evidence", {}).get("status") for c in cases if "evaluation" in c
                                   for comp in c["evaluation"]["components"] for r in comp["recommendations"]} - {None}),
               "coverage": sorted({c["evaluation"]["coverage"]["status"] for c in cases if "evaluation" in c}),
               "raises": [c["raises"][:60] for c in cases if "raises" in c]}
    print(len(cases), "cases;", json.dumps(reached, indent=1))


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit("usage: make_evaluation_golden.py <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
