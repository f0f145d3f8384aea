"""Scenario builders for analysis parity tests (runner-style trial records).

Each builder returns one trial record exercising a branch of the reference's
analysis (powermodeling/analysis.py): counter and trapezoid energy, counter
resets and disagreement, gaps, short plateaus, idle drift, clock and thermal
state checks, process inventories, epoch parsing and the paired active
reference in both orders.  They are plain data; no analysis code runs here.
"""
from __future__ import annotations

import copy
import math

BASE_POLICY = None  # the reference defaults


def _samples(start, end, hz, power, counter0=0.0, counter="float", **extra):
    out = []
    n = int(round((end - start) * hz)) + 1
    for i in range(n):
        t = start + i / hz
        s = {"t_s": t, "power_w": power(t) if callable(power) else power,
             "graphics_clock_mhz": 1200, "sm_clock_mhz": 1200, "memory_clock_mhz": 1593, "temperature_c": 50,
             "throttle_reasons": 0, "power_limit_w": 400.0, "enforced_power_limit_w": 400.0, "pstate": 0,
             "compute_processes": [], "graphics_processes": []}
        if counter == "float":
            s["energy_mj"] = (counter0 + (power(t) if callable(power) else power) * (t - start)) * 1000
        elif counter == "int":
            s["energy_mj"] = int(round((counter0 + (power if not callable(power) else power(t)) * (t - start)) * 1000))
        s.update(extra)
        out.append(s)
    return out


def steady(workload="tensor", active=150.0, idle_pre=50.0, idle_post=50.0, counter="float", hz=4,
           ops_per_s=1e12, epochs=True, pid=777, repeat=0, trial_id="steady-0", **config):
    """idle_pre 6 s, measure 12 s, idle_post 6 s with 1 s epochs (reference default windows)."""
    phases, acc = {}, 0.0
    for name, start, end, power in (("idle_pre", 0.0, 6.0, idle_pre), ("measure", 6.0, 18.0, active),
                                    ("idle_post", 18.0, 24.0, idle_post)):
        samples = _samples(start, end, hz, power, acc, counter)
        if name == "measure":
            for s in samples:
                s["compute_processes"] = [{"pid": pid, "used_gpu_memory_bytes": None}]
        phases[name] = {"start_s": start, "end_s": end, "samples": samples}
        acc += power * (end - start)
    memory = workload in ("l1", "l2", "hbm")
    bench = {"duration_s": 12.0, "operations": ops_per_s * 12, "logical_bytes": ops_per_s * 12 if memory else 0.0,
             "blocks": 80, "threads": 256, "batch_launches": 16, "iterations_per_launch": 1024}
    if epochs:
        bench["measure_epochs"] = [{"start_s": float(t), "end_s": float(t + 1), "operations": ops_per_s,
                                    "logical_bytes": ops_per_s if memory else 0.0, "counts_exact": True}
                                   for t in range(6, 18)]
    cfg = {"gpu_uuid": "GPU-golden", "graphics_clock_mhz": 1200, "memory_clock_mhz": 1593, "blocks": 80,
           "repeat": repeat}
    cfg.update(config)
    return {"trial_id": trial_id, "workload": workload, "status": "complete", "repeat": repeat, "config": cfg,
            "benchmark": bench, "phases": phases, "quality": {"measurement_pid": pid},
            "device": {"name": "Scenario fixture, not measured hardware", "power_limit_w": 400.0}}


def with_reference(record, order="AB", reference_power=80.0):
    """Add a paired active_reference arm of equal length, shifting arms for the order."""
    r = copy.deepcopy(record)
    ref_phase = copy.deepcopy(r["phases"]["measure"])
    for s in ref_phase["samples"]:
        s["power_w"] = reference_power
        s.pop("energy_mj", None)
    for p in r["phases"].values():
        for s in p["samples"]:
            s.pop("energy_mj", None)
    bench = r["benchmark"]
    ref_bench = copy.deepcopy(bench)
    ref_bench.update(operations=0, logical_bytes=0, sanity={"requested_sm_coverage_complete": True})
    for e in ref_bench.get("measure_epochs", []):
        e.update(operations=0, logical_bytes=0)
    shifted = "measure" if order == "AB" else "active_reference"
    r["phases"]["active_reference"] = ref_phase
    moved = [shifted, "idle_post"]
    for name in moved:
        p = r["phases"][name]
        p["start_s"] += 12
        p["end_s"] += 12
        for s in p["samples"]:
            s["t_s"] += 12
    for e in (bench if order == "AB" else ref_bench).get("measure_epochs", []):
        e["start_s"] += 12
        e["end_s"] += 12
    r["active_reference"] = ref_bench
    r["treatment_protocol"] = {"kind": "paired_active_reference", "order": order, "same_process": True,
                               "same_allocations": True, "same_clock_policy": True, "launch_geometry_matched": True,
                               "reference_kind": "issue_loop", "reference_workload": "control"}
    return r


def scenarios():
    """(name, record, policy) triples; policy None means the reference defaults."""
    out = []
    add = lambda name, rec, pol=None: out.append((name, rec, pol))  # noqa: E731
    add("steady_float_counter", steady())
    add("no_counter_trapezoid", steady(workload="l2", counter=None))
    r = steady(counter="int")
    for p in r["phases"].values():
        for s in p["samples"]:
            s["energy_mj"] += 1 << 60
    add("uint64_counter_offset", r)
    r = steady(counter="int")
    for s in r["phases"]["measure"]["samples"][20:]:
        s["energy_mj"] -= 500_000
    add("counter_reset", r)
    r = steady()
    for p in r["phases"].values():
        for s in p["samples"]:
            s["energy_mj"] *= 1.5
    add("counter_disagreement", r)
    r = steady()
    r["phases"]["measure"]["end_s"] = 11.0
    r["phases"]["measure"]["samples"] = [s for s in r["phases"]["measure"]["samples"] if s["t_s"] <= 11.5]
    r["benchmark"]["measure_epochs"] = [e for e in r["benchmark"]["measure_epochs"] if e["end_s"] <= 11]
    add("short_plateau", r)
    r = steady()
    r["phases"]["measure"]["samples"] = [s for s in r["phases"]["measure"]["samples"] if not 10.0 < s["t_s"] < 13.5]
    add("telemetry_gap", r)
    add("idle_drift", steady(idle_post=60.0))
    add("linear_idle_drift", steady(idle_post=54.0))
    r = steady()
    for s in r["phases"]["measure"]["samples"][10:14]:
        s["throttle_reasons"] = 4
    add("active_throttling", r)
    r = steady()
    for s in r["phases"]["measure"]["samples"][:6]:
        s["throttle_reasons"] = "0x2"
    r["phases"]["idle_pre"]["samples"][3]["throttle_reasons"] = "junk"
    add("string_throttle_masks", r)
    r = steady()
    r["phases"]["measure"]["samples"][15]["compute_processes"].append({"pid": 9999})
    add("foreign_process", r)
    r = steady()
    r["phases"]["idle_pre"]["samples"][8]["graphics_processes"] = None
    add("missing_inventory", r)
    r = steady()
    for p in r["phases"].values():
        for s in p["samples"]:
            s["graphics_clock_mhz"] = 1100
    add("clock_mismatch", r)
    r = steady()
    for i, s in enumerate(r["phases"]["measure"]["samples"]):
        s["graphics_clock_mhz"] = 1150 + (i % 3) * 50
    add("clock_drift", r)
    r = steady()
    for i, s in enumerate(r["phases"]["measure"]["samples"]):
        s["temperature_c"] = 50 + i * 0.25
    add("temperature_drift_and_idle_mismatch", r)
    r = steady()
    for s in r["phases"]["idle_pre"]["samples"]:
        s["pstate"] = 8
        s["graphics_clock_mhz"] = 900
    add("idle_pstate_and_downclock", r)
    add("paired_ab", with_reference(steady(workload="l2", counter=None), "AB"))
    add("paired_ba", with_reference(steady(workload="l2", counter=None), "BA"))
    add("paired_tensor_ab", with_reference(steady(counter=None), "AB", reference_power=100.0))
    add("paired_negative_contrast", with_reference(steady(workload="l2", counter=None), "AB", reference_power=170.0))
    r = with_reference(steady(workload="l2", counter=None), "BA")
    for s in r["phases"]["active_reference"]["samples"][5:9]:
        s["graphics_clock_mhz"] = 1500
    r["phases"]["active_reference"]["samples"][2]["compute_processes"] = [{"pid": None}]
    add("paired_state_mismatch", r)
    r = steady(epochs=False)
    r["benchmark"]["host_duration_s"] = 12.2
    add("legacy_no_epochs", r)
    r = steady()
    r["benchmark"]["measure_epochs"][3]["start_s"] = 8.5
    add("overlapping_epochs", r)
    r = steady()
    r["benchmark"]["measure_epochs"][0]["start_s"] = 5.0
    add("epoch_outside_window", r)
    r = steady()
    r["benchmark"]["measure_epochs"].append("not an epoch")
    add("non_dict_epoch", r)
    r = steady()
    r["benchmark"]["operations"] *= 1.01
    add("epoch_total_disagreement", r)
    r = steady()
    r["benchmark"]["measure_epochs"] = []
    add("empty_epoch_list", r)
    r = steady()
    for e in r["benchmark"]["measure_epochs"]:
        e["host_monotonic_start_ns"] = int(e.pop("start_s") * 1e9)
        e["host_monotonic_end_ns"] = int(e.pop("end_s") * 1e9)
    r["benchmark"]["measure_epochs"].reverse()
    add("ns_epochs_unsorted", r)
    r = steady()
    samples = r["phases"]["measure"]["samples"]
    dup = copy.deepcopy(samples[10])
    dup["power_w"] = 900.0
    samples.insert(3, dup)
    samples.reverse()
    add("duplicate_and_unsorted_timestamps", r)
    r = steady(counter=None)
    r["phases"]["measure"]["samples"][12]["power_w"] = None
    r["phases"]["idle_pre"]["samples"][4]["power_w"] = True
    r["phases"]["idle_post"]["samples"][5]["temperature_c"] = "51"
    add("none_bool_and_string_values", r)
    r = steady(counter=None)
    r["phases"]["idle_post"]["samples"][2]["power_w"] = -3.0
    add("negative_idle_power", r)
    r = steady()
    for p, level in (("idle_pre", 20.0), ("measure", 40.0), ("idle_post", 20.0)):
        for s in r["phases"][p]["samples"]:
            s["memory_power_w"] = level
            s["memory_power_source"] = "memory_power_instant_w"
    add("memory_rail", r)
    r = steady(trial_id="")
    r["quality"]["valid"] = False
    r["status"] = "failed"
    add("runner_quality_and_status", r)
    r = steady()
    r["cuda_device"] = {"compute_capability": "9.0", "sm_count": 132, "name": "NVIDIA H100 80GB HBM3"}
    add("tensor_peak_h100", r)
    r = steady()
    for p in r["phases"].values():
        for s in p["samples"]:
            s.pop("sm_clock_mhz", None)
    r["cuda_device"] = {"compute_capability": [8, 0], "sm_count": 108}
    add("tensor_peak_graphics_proxy", r)
    r = steady()
    r["phases"]["active_control"] = copy.deepcopy(r["phases"]["measure"])
    for s in r["phases"]["active_control"]["samples"]:
        s["power_w"] = 70.0
    add("active_control_descriptive", r)
    r = steady()
    del r["phases"]["idle_post"]
    add("missing_idle_post", r)
    r = steady()
    r["phases"]["measure"]["start_s"] = None
    add("invalid_measure_window", r)
    short = dict(trim_s=0.0, idle_trim_s=0.0, min_measure_s=1.0, min_idle_s=0.5)
    add("short_policy_steady", steady(), short)
    return out
