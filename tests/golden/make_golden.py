"""Generate the golden analysis fixtures from the reference implementation.

Run in a checkout where the reference package is importable (read-only):
    python tests/golden/make_golden.py <reference checkout>      (or PM_REFERENCE_TREE=<reference checkout>)
It imports powermodeling.analysis from that tree, runs the reference's own
analyze_trial / summarize / _median_ci on inputs rebuilt deterministically
by tests/trial_builders.py and powermodeling_b200.synthetic, and writes their
outputs to tests/golden/*.json.gz.  The inputs are not stored: tests rebuild
them and check a digest, so the fixtures hold only reference outputs.
B = 10 000 intervals use the reference's _median_ci generalised to B draws
with order statistics 25B/1000-1 and 975B/1000-1 (B = 1000 gives [24], [974]).
"""
from __future__ import annotations

import gzip
import hashlib
import json
import math
import random
import statistics
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

TRIAL_KEYS = (
    "valid", "issues", "warnings", "baseline_valid", "baseline_issues", "duration_s", "benchmark_duration_s",
    "count_energy_time_alignment_exact", "counted_measure_operations", "counted_measure_logical_bytes",
    "complete_measure_epochs", "throughput_ops_s", "throughput_bytes_s", "device_event_throughput_ops_s",
    "board_power_w", "idle_power_w", "incremental_power_w", "operational_idle_increment_energy_j",
    "operational_idle_increment_eligible", "total_energy_j", "idle_energy_j", "incremental_energy_j",
    "integrated_power_energy_j", "energy_counter_j", "energy_source", "pj_per_op", "pj_per_logical_byte",
    "total_pj_per_op", "total_pj_per_logical_byte", "total_pj_per_flop", "total_pj_per_logical_bit",
    "operational_idle_increment_pj_per_flop", "operational_idle_increment_pj_per_logical_bit",
    "memory_rail_power_w", "memory_rail_idle_power_w", "memory_rail_energy_j", "memory_rail_incremental_energy_j",
    "memory_rail_incremental_power_w", "graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz", "temperature_c",
    "throttle_reasons_mask", "other_gpu_process_pids", "power_limit_w", "idle_fraction_of_measured_power",
    "idle_fraction_of_power_limit", "power_limit_utilization", "tensor_peak_tflops_at_achieved_clock",
    "tensor_peak_clock_source", "tensor_utilization_vs_dense_clock_peak",
    "baseline_clock_matched", "baseline_temperature_matched", "baseline_power_cap_matched", "baseline_state_matched",
    "baseline_state_issues", "active_minus_idle_state_deltas", "paired_active_reference_eligible",
    "paired_active_reference_power_w", "paired_active_reference_energy_j", "paired_active_reference_issues",
    "paired_active_reference_pj_per_flop", "paired_active_reference_pj_per_logical_bit",
    "paired_active_reference_drift_adjusted_power_w", "active_reference_power_w", "active_reference_duration_s",
    "active_reference_total_energy_j", "paired_active_reference_state_deltas", "active_control_incremental_power_w",
    "throughput_elements_s", "throughput_rows_s", "counted_measure_elements", "row_width", "total_pj_per_element",
    "total_pj_per_row", "operational_idle_increment_pj_per_element", "operational_idle_increment_pj_per_row",
    "paired_active_reference_pj_per_element", "paired_active_reference_pj_per_row",
)
PHASE_KEYS = ("issues", "warnings", "start_s", "end_s", "duration_s", "midpoint_s", "samples",
              "sample_interval_median_s", "max_sample_gap_s", "integrated_power_energy_j", "integrated_power_w",
              "power_w", "memory_rail_energy_j", "memory_power_w", "energy_counter_j",
              "counter_power_disagreement_fraction", "distinct_power_values",
              "observed_power_change_interval_median_s", "graphics_clock_mhz", "graphics_clock_mhz_min",
              "graphics_clock_mhz_max", "sm_clock_mhz", "memory_clock_mhz", "temperature_c", "temperature_c_min",
              "temperature_c_max")


def records_digest(records) -> str:
    return hashlib.sha256(json.dumps(records, sort_keys=True, default=str).encode()).hexdigest()


def pick(trial: dict) -> dict:
    out = {k: trial.get(k) for k in TRIAL_KEYS if k in trial}
    out["phases"] = {name: {k: p.get(k) for k in PHASE_KEYS if k in p} for name, p in trial.get("phases", {}).items()}
    return out


def generalised_median_ci(values, seed, resamples):
    rng = random.Random(seed)
    draws = sorted(statistics.median(rng.choices(values, k=len(values))) for _ in range(resamples))
    return [draws[25 * resamples // 1000 - 1], draws[975 * resamples // 1000 - 1]]


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling import analysis as ref  # the reference implementation
    from trial_builders import scenarios
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep

    cases = []
    for name, record, policy in scenarios():
        trial = ref.analyze_trial(record, policy)
        cases.append({"name": name, "policy": policy, "digest": records_digest([record]), "expected": pick(trial)})
    sweeps = []
    for label, shape, seed in (("sweep_trapezoid", SweepShape(points=3, repeats=4), 11),
                               ("sweep_counter", SweepShape(points=2, repeats=4, with_energy_counter=True), 12),
                               ("sweep_five_repeats", SweepShape(points=2, repeats=5), 13)):
        records = make_sweep(shape, seed)
        summary = ref.summarize(records, policy=ANALYSIS_POLICY)
        groups = [{"group_id": g["group_id"], "valid_repeats": g["valid_repeats"], "trial_ids": g["trial_ids"],
                   "medians": {m: g.get(m) for m in ref._METRICS}, "ci95": {m: g["ci95"].get(m) for m in ref._METRICS},
                   "paired_reference_order_counts": g["paired_reference_order_counts"],
                   "paired_active_reference_eligible": g["paired_active_reference_eligible"],
                   "paired_reference_order_effect_power_w": g["paired_reference_order_effect_power_w"]}
                  for g in summary["groups"]]
        sweeps.append({"name": label, "shape": shape.__dict__, "seed": seed, "digest": records_digest(records),
                       "trials": [pick(t) for t in summary["trials"]], "groups": groups,
                       "group_keys": [ref._group_key(t) for t in summary["trials"]]})
    rng = random.Random(2024)
    seeds = [0, 1, 7, 2 ** 32 - 1, 2 ** 32, 2 ** 63 + 5, 2 ** 64 - 1,
             int(hashlib.sha256(b"b200").hexdigest()[:16], 16), int(hashlib.sha256(b"group").hexdigest()[:16], 16)]
    ci_cases = []
    for seed in seeds:
        for n in (3, 4, 5, 6, 7, 8, 11, 20):
            values = [round(rng.uniform(-5, 500), rng.choice([0, 3, 9])) for _ in range(n)]
            if n == 6:
                values[2] = values[4]          # ties
            ci_cases.append({"seed": seed, "values": values, "ci_1000": ref._median_ci(values, seed),
                             "ci_10000": generalised_median_ci(values, seed, 10000)})
    streams = []
    for seed in seeds[:6]:
        for n in (3, 4, 9):
            r = random.Random(seed)
            streams.append({"seed": seed, "n": n, "rows": [r.choices(range(n), k=n) for _ in range(40)]})
    HERE.mkdir(parents=True, exist_ok=True)
    for filename, payload in (("analysis_trials.json.gz", {"trial_keys": TRIAL_KEYS, "phase_keys": PHASE_KEYS, "cases": cases}),
                              ("analysis_sweeps.json.gz", {"sweeps": sweeps}),
                              ("median_ci.json.gz", {"cases": ci_cases, "streams": streams})):
        with gzip.open(HERE / filename, "wt") as f:
            json.dump(payload, f, allow_nan=True, separators=(",", ":"))
        print("wrote", filename)


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit(f"usage: {Path(__file__).name} <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
