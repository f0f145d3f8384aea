"""NVML memory-scope (HBM rail) observations qualified independently of device power.

Restates powermodeling/memory_power.py: ``phase_sensor`` (27-123) checks
precisely the samples that cover one integration window — sensor source,
scope, field and semantics metadata, sensor-timestamp freshness and order,
latency, gaps, sign — ``trial_sensor`` (126-166) turns the measure window
into energy, normalised and idle-incremental figures, and ``group_sensor``
(169-204) takes repeat medians and bootstrap intervals.

The numbers come from the GPU path: the window energy is the analysis
kernel's memory-rail trapezoid for the phase (the same samples and the same
interpolation at the window edges the reference integrates), and the group
intervals come from the bootstrap kernel, run on extra columns holding each
repeat's sensor fields.  The per-sample checks are host logic over the
sample dictionaries, like the reference's.
"""
from __future__ import annotations

import math
import statistics
from typing import Any, Mapping

SOURCES = {
    "memory_power_instant_w": ("driver_instantaneous", "NVML_FI_DEV_POWER_INSTANT"),
    "memory_power_average_w": ("one_second_average", "NVML_FI_DEV_POWER_AVERAGE"),
}
NUMERIC_FIELDS = ("power_w", "energy_j", "idle_power_w", "incremental_power_w",
                  "incremental_energy_j", "pj_per_logical_bit", "incremental_pj_per_logical_bit")
ALIASES = (("memory_rail_power_w", "power_w"), ("memory_rail_energy_j", "energy_j"),
           ("memory_rail_idle_power_w", "idle_power_w"),
           ("memory_rail_incremental_power_w", "incremental_power_w"),
           ("memory_rail_incremental_energy_j", "incremental_energy_j"))


def number(value: Any) -> float | None:
    return float(value) if isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value) else None


def empty() -> dict[str, Any]:
    return {"status": "unavailable", "scope": "memory", "source": None,
            "semantics": None, **dict.fromkeys(NUMERIC_FIELDS),
            "measurement_valid": False, "normalization_valid": False,
            "incremental_valid": False, "issues": [], "incremental_issues": [],
            "freshness_verified": False, "freshness_status": "unverified",
            "maximum_sensor_age_s": None, "freshness_maximum_age_s": None}


def _covering(samples: list[dict], start: float, end: float) -> list[dict]:
    """Samples inside [start, end], widened by one neighbour on a side that does not reach its edge."""
    covering = [s for s in samples if start <= s["t_s"] <= end]
    if not covering or covering[0]["t_s"] != start:
        before = [s for s in samples if s["t_s"] < start]
        covering = before[-1:] + covering
    if not covering or covering[-1]["t_s"] < end:
        after = [s for s in samples if s["t_s"] > end]
        covering += after[:1]
    return covering


def phase_sensor(phase: Mapping | None, stats: Mapping, maximum_gap: float, energy: float | None) -> dict[str, Any]:
    """One window's memory-rail reading; ``energy`` is the kernel's trapezoid of memory_power_w over it."""
    result = empty()
    by_time = {number(s.get("t_s")): s for s in (phase or {}).get("samples", [])
               if isinstance(s, dict) and number(s.get("t_s")) is not None}
    samples = [by_time[t] for t in sorted(by_time)]
    start, end = number(stats.get("start_s")), number(stats.get("end_s"))
    if start is None or end is None or end <= start:
        result["issues"] = ["invalid_memory_sensor_window"]
        result["status"] = "invalid" if any(s.get("memory_power_w") is not None for s in samples) else "unavailable"
        return result
    covering = _covering(samples, start, end)
    if not any(s.get("memory_power_w") is not None for s in covering):
        result["issues"] = ["memory_sensor_unavailable"]
        return result
    issues = []
    if not covering or covering[0]["t_s"] > start or covering[-1]["t_s"] < end:
        issues.append("missing_memory_sensor_coverage")
    values = [number(s.get("memory_power_w")) for s in covering]
    if any(v is None for v in values):
        issues.append("missing_memory_sensor_coverage")
    if any(v is not None and v < 0 for v in values):
        issues.append("negative_memory_sensor_power")
    if any(b["t_s"] - a["t_s"] > maximum_gap for a, b in zip(covering, covering[1:])):
        issues.append("memory_sensor_telemetry_gap")
    sources = {s.get("memory_power_source") for s in covering}
    if any(source not in SOURCES for source in sources):
        issues.append("unknown_memory_sensor_source")
    if len(sources) != 1:
        issues.append("mixed_memory_sensor_sources")
    source = next(iter(sources)) if len(sources) == 1 else None
    source = source if source in SOURCES else None
    result["source"] = source
    result["semantics"] = SOURCES[source][0] if source else None
    timestamps, ages = [], []
    comparable = 0
    # A one-second average may repeat between updates: a stale-reading bound, not a refresh cadence.
    maximum_age = max(1.5, maximum_gap)
    result["freshness_maximum_age_s"] = maximum_age
    for sample in covering:
        selected = sample.get("memory_power_source")
        errors = sample.get("errors") or {}
        if errors.get("memory_power_w") or selected and errors.get(selected):
            issues.append("memory_sensor_query_error")
        metadata = (sample.get("field_metadata") or {}).get(selected)
        if metadata is None:
            continue
        if not isinstance(metadata, dict) or metadata.get("scope") != "memory":
            issues.append("invalid_memory_sensor_scope")
            continue
        expected = SOURCES.get(selected)
        if expected and ("field" in metadata and metadata["field"] != expected[1] or
                         "semantics" in metadata and metadata["semantics"] != expected[0]):
            issues.append("inconsistent_memory_sensor_metadata")
        if "timestamp_us" in metadata:
            timestamp = number(metadata["timestamp_us"])
            if timestamp is None or timestamp < 0:
                issues.append("invalid_memory_sensor_timestamp")
            else:
                timestamps.append(timestamp)
                clock = metadata.get("timestamp_clock")
                if clock is not None and clock != "unix_epoch_microseconds":
                    issues.append("invalid_memory_sensor_timestamp_clock")
                q0, q1 = number(sample.get("query_realtime_start_s")), number(sample.get("query_realtime_end_s"))
                if clock == "unix_epoch_microseconds" and q0 is not None and q1 is not None:
                    if q1 < q0:
                        issues.append("invalid_memory_sensor_query_timestamps")
                    else:
                        comparable += 1
                        field_time = timestamp / 1e6
                        age = max(0.0, q0 - field_time)
                        ages.append(age)
                        if age > maximum_age:
                            issues.append("stale_memory_sensor_timestamp")
                        if field_time > q1 + .001:
                            issues.append("future_memory_sensor_timestamp")
        if "latency_us" in metadata and (number(metadata["latency_us"]) is None or metadata["latency_us"] < 0):
            issues.append("invalid_memory_sensor_latency")
    if any(b < a for a, b in zip(timestamps, timestamps[1:])):
        issues.append("memory_sensor_timestamp_regression")
    result["maximum_sensor_age_s"] = max(ages) if ages else None
    result["freshness_status"] = ("verified" if comparable == len(covering) else "partial" if comparable
                                  else "unverified")
    result["freshness_verified"] = comparable == len(covering) and not issues
    if comparable and issues:
        result["freshness_status"] = "invalid"
    if energy is None:
        issues.append("missing_memory_sensor_coverage")
    result["issues"] = sorted(set(issues))
    result["status"] = "invalid" if issues else "available"
    result["measurement_valid"] = not issues
    if not issues:
        result["energy_j"] = energy
        result["power_w"] = energy / (end - start)
    return result


def _idle_at(pre: Mapping, post: Mapping, active: Mapping, field: str) -> float | None:
    """Idle level interpolated at the active window's midpoint (analysis.py:210-216)."""
    a, b = number(pre.get(field)), number(post.get(field))
    t0, t1, t = number(pre.get("midpoint_s")), number(post.get("midpoint_s")), number(active.get("midpoint_s"))
    if any(v is None for v in (a, b, t0, t1, t)) or t1 <= t0 or not t0 <= t <= t1:
        return None
    return a + (b - a) * (t - t0) / (t1 - t0)


def trial_sensor(record: Mapping, result: Mapping, phases: Mapping, phase_records: Mapping,
                 maximum_gap: float, maximum_idle_drift: float) -> dict[str, Any] | None:
    """Memory-rail record of one HBM trial (memory_power.py:126-166)."""
    if record.get("workload") != "hbm":
        return None
    energy = lambda name: number(phases[name].get("memory_rail_energy_j"))  # noqa: E731
    sensor = phase_sensor(phase_records.get("measure"), phases["measure"], maximum_gap, energy("measure"))
    count = number(result.get("counted_measure_logical_bytes"))
    exact = result.get("count_energy_time_alignment_exact") is True
    sensor["normalization_valid"] = bool(sensor["measurement_valid"] and result.get("valid") and exact
                                         and count is not None and count > 0)
    if sensor["normalization_valid"]:
        sensor["pj_per_logical_bit"] = sensor["energy_j"] / (count * 8) * 1e12
    pre = phase_sensor(phase_records.get("idle_pre"), phases["idle_pre"], maximum_gap, energy("idle_pre"))
    post = phase_sensor(phase_records.get("idle_post"), phases["idle_post"], maximum_gap, energy("idle_post"))
    incremental_issues = ["idle_pre:" + issue for issue in pre["issues"]]
    incremental_issues += ["idle_post:" + issue for issue in post["issues"]]
    if sensor["source"] is None or pre["source"] != sensor["source"] or post["source"] != sensor["source"]:
        incremental_issues.append("idle_memory_sensor_source_mismatch")
    if not incremental_issues:
        idle = _idle_at({**phases["idle_pre"], "memory_power_w": pre["power_w"]},
                        {**phases["idle_post"], "memory_power_w": post["power_w"]},
                        phases["measure"], "memory_power_w")
        if idle is None:
            incremental_issues.append("missing_idle_memory_sensor_baseline")
        else:
            sensor["idle_power_w"] = idle
            drift = abs(pre["power_w"] - post["power_w"]) / max((pre["power_w"] + post["power_w"]) / 2, 1e-9)
            if drift > maximum_idle_drift:
                incremental_issues.append("memory_idle_baseline_drift")
    if not sensor["measurement_valid"]:
        incremental_issues.append("invalid_treatment_memory_sensor")
    if result.get("operational_idle_increment_eligible") is not True:
        incremental_issues.append("unqualified_matched_idle_baseline")
    if not incremental_issues:
        sensor["incremental_power_w"] = sensor["power_w"] - sensor["idle_power_w"]
        sensor["incremental_energy_j"] = sensor["energy_j"] - sensor["idle_power_w"] * result["duration_s"]
        sensor["incremental_valid"] = True
        if sensor["normalization_valid"]:
            sensor["incremental_pj_per_logical_bit"] = sensor["incremental_energy_j"] / (count * 8) * 1e12
    sensor["incremental_issues"] = sorted(set(incremental_issues))
    return sensor


def bootstrap_columns(sensor: Mapping | None) -> list[float]:
    """One repeat's values of NUMERIC_FIELDS for the group bootstrap, NaN outside each field's population."""
    nan = float("nan")
    if not sensor or not sensor["measurement_valid"]:
        return [nan] * len(NUMERIC_FIELDS)
    out = []
    for field in NUMERIC_FIELDS:
        member = (sensor["normalization_valid"] if field == "pj_per_logical_bit"
                  else sensor["incremental_valid"] if field.startswith("incremental_") else True)
        value = number(sensor[field]) if member else None
        out.append(nan if value is None else value)
    return out


def group_sensor(trials: list, workload: str, observed_trials: list | None,
                 medians: list, intervals: list) -> dict[str, Any] | None:
    """Repeat medians and intervals of the memory-rail fields (memory_power.py:169-204).

    ``medians``/``intervals`` hold, per NUMERIC_FIELDS entry, the median and
    the [lo, hi] interval the bootstrap kernel computed over
    ``bootstrap_columns`` of the group's valid repeats.
    """
    if workload != "hbm":
        return None
    result = empty()
    observed = trials if observed_trials is None else observed_trials
    sensors = [trial["hbm_memory_power"] for trial in trials]
    measured = [s for s in sensors if s["measurement_valid"]]
    normalized = [s for s in measured if s["normalization_valid"]]
    incremental = [s for s in measured if s["incremental_valid"]]
    excluded_invalid = sum(trial.get("valid") is not True for trial in observed)
    excluded_duplicate = len(observed) - len(trials) - excluded_invalid
    result.update(observed_repeats=len(observed), valid_repeats=len(measured),
                  normalized_repeats=len(normalized), incremental_repeats=len(incremental),
                  board_invalid_repeats=excluded_invalid, duplicate_repeats_excluded=excluded_duplicate,
                  ci95=dict.fromkeys(NUMERIC_FIELDS))
    result["issues"] = sorted({issue for s in sensors for issue in s["issues"]})
    if excluded_invalid:
        result["issues"].append("board_invalid_repeats_excluded")
    if excluded_duplicate:
        result["issues"].append("duplicate_repeat_indices_excluded")
    result["incremental_issues"] = sorted({issue for s in sensors for issue in s["incremental_issues"]})
    sources = {s["source"] for s in measured}
    if len(sources) > 1:
        result["status"] = "invalid"
        result["issues"] = sorted(set(result["issues"] + ["mixed_memory_sensor_sources_across_repeats"]))
        return result
    if not measured:
        all_board_invalid = bool(observed) and excluded_invalid == len(observed)
        result["status"] = "invalid" if all_board_invalid or any(s["status"] == "invalid" for s in sensors) else "unavailable"
        return result
    result.update(status="available" if len(measured) == len(observed) else "partial",
                  source=measured[0]["source"], semantics=measured[0]["semantics"],
                  measurement_valid=True, normalization_valid=bool(normalized), incremental_valid=bool(incremental))
    result["freshness_verified"] = all(s["freshness_verified"] for s in measured)
    result["freshness_status"] = ("verified" if result["freshness_verified"] else "partial"
                                  if any(s["freshness_status"] != "unverified" for s in measured) else "unverified")
    result["maximum_sensor_age_s"] = max((s["maximum_sensor_age_s"] for s in measured
                                          if s["maximum_sensor_age_s"] is not None), default=None)
    result["freshness_maximum_age_s"] = min(s["freshness_maximum_age_s"] for s in measured)
    for k, field in enumerate(NUMERIC_FIELDS):
        result[field] = medians[k]
        result["ci95"][field] = intervals[k]
    return result


def host_median(values: list[float]) -> float | None:
    """statistics.median of the finite values (used where a group has no bootstrap columns)."""
    vals = [v for v in values if v is not None]
    return statistics.median(vals) if vals else None
