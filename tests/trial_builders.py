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


def nonlinear_steady(workload="rmsnorm", batches_per_epoch=50, **kw):
    """steady() carrying a Q-grid result of a complete nonlinear function
    (the record shape of powerbench's exp|tanh|silu|rmsnorm|softmax arms), one
    epoch per second of the 12 s measure window."""
    from nonlinear_cases import q_grid_record
    r = steady(workload=workload, **kw)
    bench = q_grid_record(workload, epoch_batches=(batches_per_epoch,) * 12)
    for k, e in enumerate(bench["measure_epochs"]):
        e.update(start_s=6.0 + k, end_s=7.0 + k)
    bench["duration_s"] = 12.0
    r["benchmark"] = bench
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
    for count in (32, 33, 48):
        # Epoch lists on both sides of the 32 a CTA copies to shared memory.
        r = steady()
        width = 12.0 / count
        r["benchmark"]["measure_epochs"] = [{"start_s": 6.0 + k * width, "end_s": 6.0 + (k + 1) * width,
                                             "operations": 1e12 * width, "logical_bytes": 0.0, "counts_exact": True}
                                            for k in range(count)]
        r["benchmark"]["measure_epochs"].reverse()
        add(f"epochs_{count}_unsorted", r)
    r = with_reference(steady(workload="l2", counter=None), "AB")
    for e_list in (r["benchmark"]["measure_epochs"], r["active_reference"]["measure_epochs"]):
        base = e_list[0]["start_s"]
        e_list[:] = [{"start_s": base + k * 0.25, "end_s": base + (k + 1) * 0.25, "operations": e_list[0]["operations"] / 4,
                      "logical_bytes": e_list[0]["logical_bytes"] / 4, "counts_exact": True} for k in range(48)]
    add("paired_48_epochs_per_arm", r)
    add("nonlinear_rmsnorm_q_grid", nonlinear_steady("rmsnorm"))
    add("nonlinear_exp_trapezoid", nonlinear_steady("exp", counter=None))
    add("nonlinear_softmax_paired_ab", with_reference(nonlinear_steady("softmax", counter=None), "AB", reference_power=90.0))
    add("nonlinear_silu_paired_ba", with_reference(nonlinear_steady("silu", counter=None), "BA", reference_power=120.0))
    r = nonlinear_steady("tanh")
    r["benchmark"]["elements"] += 1
    add("nonlinear_count_disagreement", r)
    r = nonlinear_steady("rmsnorm")
    r["benchmark"]["sanity"]["numerical_validation_passed"] = False
    add("nonlinear_validation_failed", r)
    return out


# ---------------------------------------------------------------- HBM memory-rail sensor cases
WALL0 = 1_764_000_000.0  # CLOCK_REALTIME of t_s = 0 in these fixtures


def memory_rail(active_memory=60.0, idle_memory=20.0, idle_post_memory=None, source="memory_power_instant_w",
                ripple=0.25, workload_override=None, **kw):
    """An HBM trial whose samples carry the NVML memory-scope power field with its sensor metadata."""
    r = steady(workload=workload_override or "hbm", **kw)
    field, semantics = (("NVML_FI_DEV_POWER_INSTANT", "driver_instantaneous") if source == "memory_power_instant_w"
                        else ("NVML_FI_DEV_POWER_AVERAGE", "one_second_average"))
    levels = {"idle_pre": idle_memory, "measure": active_memory,
              "idle_post": idle_memory if idle_post_memory is None else idle_post_memory}
    for name, phase in r["phases"].items():
        for k, s in enumerate(phase["samples"]):
            t = s["t_s"]
            s["memory_power_w"] = levels[name] + ripple * ((k * 7) % 5 - 2)
            s["memory_power_source"] = source
            s["query_realtime_start_s"] = WALL0 + t - 0.001
            s["query_realtime_end_s"] = WALL0 + t + 0.001
            s["errors"] = {}
            s["field_metadata"] = {source: {"field": field, "scope": "memory", "scope_id": 2,
                                            "timestamp_us": int(round((WALL0 + t - 0.004) * 1e6)),
                                            "timestamp_clock": "unix_epoch_microseconds", "latency_us": 20,
                                            "semantics": semantics}}
    return r


def _measure_samples(r):
    return r["phases"]["measure"]["samples"]


def memory_rail_scenarios():
    """(name, record) pairs for the memory-rail sensor (memory_power.py:27-166)."""
    out = [("fresh", memory_rail()), ("average_source", memory_rail(source="memory_power_average_w"))]
    r = memory_rail()
    for s in _measure_samples(r)[10:14]:
        s["field_metadata"][s["memory_power_source"]]["timestamp_us"] -= 3_000_000
    out.append(("stale_timestamps", r))
    r = memory_rail()
    _measure_samples(r)[12]["field_metadata"]["memory_power_instant_w"]["timestamp_us"] += 2_000_000
    out.append(("future_timestamp", r))
    r = memory_rail()
    for s in r["phases"]["idle_post"]["samples"]:
        s["memory_power_source"] = "memory_power_average_w"
        s["field_metadata"] = {"memory_power_average_w": dict(s["field_metadata"]["memory_power_instant_w"],
                                                              field="NVML_FI_DEV_POWER_AVERAGE",
                                                              semantics="one_second_average")}
    out.append(("idle_source_mismatch", r))
    r = memory_rail()
    _measure_samples(r)[13]["memory_power_source"] = "memory_power_module_w"
    out.append(("unknown_source", r))
    r = memory_rail()
    _measure_samples(r)[9]["field_metadata"]["memory_power_instant_w"]["scope"] = "gpu"
    out.append(("wrong_scope", r))
    r = memory_rail()
    _measure_samples(r)[11]["field_metadata"]["memory_power_instant_w"]["semantics"] = "one_second_average"
    out.append(("inconsistent_metadata", r))
    r = memory_rail()
    meta = [s["field_metadata"]["memory_power_instant_w"] for s in _measure_samples(r)]
    meta[20]["timestamp_us"], meta[21]["timestamp_us"] = meta[21]["timestamp_us"], meta[20]["timestamp_us"]
    out.append(("timestamp_regression", r))
    r = memory_rail()
    _measure_samples(r)[15]["memory_power_w"] = None
    out.append(("missing_value", r))
    r = memory_rail()
    _measure_samples(r)[16]["memory_power_w"] = -1.0
    out.append(("negative_power", r))
    r = steady(workload="hbm")
    out.append(("no_memory_sensor", r))
    r = memory_rail()
    _measure_samples(r)[14]["errors"] = {"memory_power_instant_w": {"type": "NVMLError_Timeout", "message": "Timeout"}}
    out.append(("query_error", r))
    r = memory_rail()
    _measure_samples(r)[17]["field_metadata"]["memory_power_instant_w"]["latency_us"] = -1
    out.append(("negative_latency", r))
    r = memory_rail()
    _measure_samples(r)[18]["field_metadata"]["memory_power_instant_w"]["timestamp_clock"] = "monotonic"
    out.append(("other_timestamp_clock", r))
    r = memory_rail()
    _measure_samples(r)[19]["query_realtime_end_s"] = _measure_samples(r)[19]["query_realtime_start_s"] - 1
    out.append(("query_clock_backwards", r))
    out.append(("idle_drift", memory_rail(idle_post_memory=30.0)))
    r = memory_rail()
    for s in _measure_samples(r):
        s["field_metadata"] = {}
    out.append(("no_metadata", r))
    r = memory_rail()
    r["phases"]["measure"]["samples"] = [s for s in _measure_samples(r) if not 10.0 < s["t_s"] < 13.5]
    out.append(("sensor_gap", r))
    r = memory_rail()
    r["benchmark"].pop("measure_epochs")
    out.append(("not_count_exact", r))
    out.append(("l2_workload_has_no_sensor", memory_rail(workload_override="l2")))
    return out


def memory_rail_group():
    """Repeats of one HBM configuration: valid, stale, drifting idle and board-invalid members."""
    reps = []
    for k, active in enumerate((60.0, 63.5, 58.25, 61.0, 59.5, 62.0)):
        reps.append(memory_rail(active_memory=active, repeat=k, trial_id=f"rail-{k}"))
    for s in _measure_samples(reps[3])[10:14]:
        s["field_metadata"][s["memory_power_source"]]["timestamp_us"] -= 3_000_000
    for s in reps[4]["phases"]["idle_post"]["samples"]:
        s["memory_power_w"] = 30.0
    reps[5]["phases"]["measure"]["samples"][15]["compute_processes"].append({"pid": 4321})
    mixed = [memory_rail(active_memory=60.0 + k, repeat=k, trial_id=f"mixed-{k}", blocks=96,
                         source="memory_power_average_w" if k == 1 else "memory_power_instant_w") for k in range(3)]
    return reps + mixed
