"""NVML memory-scope (HBM rail) observations qualified independently of device power.

The memory rail's energy over a window comes from the GPU path (the analysis
kernel's memory-rail trapezoid, with the same samples and edge
interpolation as the board-power integral); the group intervals come from
the bootstrap kernel, run on extra columns holding each repeat's sensor
fields.  This module qualifies those numbers: every sample that covers an
integration window is inspected on its own (``_inspect``: the value, the
query errors, the field's scope, source and semantics metadata, the sensor
timestamp's clock, age and order), the window as a whole is checked for
coverage, gaps and a single known source (``WINDOW_RULES``), and the
trial and group records are assembled from the qualified windows.  Issue
strings, record keys and the rules they name are the reference's
(powermodeling/memory_power.py: windows 27-123, trials 126-166, groups
169-204), pinned by fixtures its own functions produced
(tests/golden/memory_power.json.gz).
"""
from __future__ import annotations

import bisect
import math
import statistics
from dataclasses import dataclass, field
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
UNIX_US = "unix_epoch_microseconds"
# A one-second average may repeat between updates: the staleness bound is on
# the reading's age, not on a refresh cadence.
MIN_STALE_AGE_S = 1.5


def number(value: Any) -> float | None:
    return float(value) if isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value) else None


def empty() -> dict[str, Any]:
    return {"status": "unavailable", "scope": "memory", "source": None,
            "semantics": None, **dict.fromkeys(NUMERIC_FIELDS),
            "measurement_valid": False, "normalization_valid": False,
            "incremental_valid": False, "issues": [], "incremental_issues": [],
            "freshness_verified": False, "freshness_status": "unverified",
            "maximum_sensor_age_s": None, "freshness_maximum_age_s": None}


# ---------------------------------------------------------------------------- one window
def _by_time(phase: Mapping | None) -> tuple[list[float], list[dict]]:
    """The phase's samples with a finite t_s, one per instant (the last wins), in time order."""
    latest: dict[float, dict] = {}
    for s in (phase or {}).get("samples", []):
        if isinstance(s, dict) and (t := number(s.get("t_s"))) is not None:
            latest[t] = s
    times = sorted(latest)
    return times, [latest[t] for t in times]


def _cover(times: list[float], samples: list[dict], start: float, end: float) -> list[dict]:
    """Samples in [start, end], plus the nearest one outside on each side the inside ones do not reach."""
    lo, hi = bisect.bisect_left(times, start), bisect.bisect_right(times, end)
    if lo == hi or times[lo] != start:
        lo = max(lo - 1, 0)
    if hi < len(times) and (lo == hi or times[hi - 1] < end):
        hi += 1
    return samples[lo:hi]


@dataclass
class _Reading:
    """What one covering sample contributes to its window's qualification."""
    issues: set = field(default_factory=set)
    timestamp: float | None = None        # the sensor's own timestamp (us), when valid
    age: float | None = None              # query start minus sensor time (s), when comparable


def _inspect(sample: Mapping, maximum_age: float) -> _Reading:
    out = _Reading()
    selected = sample.get("memory_power_source")
    errors = sample.get("errors") or {}
    if errors.get("memory_power_w") or selected and errors.get(selected):
        out.issues.add("memory_sensor_query_error")
    meta = (sample.get("field_metadata") or {}).get(selected)
    if meta is None:
        return out
    if not isinstance(meta, dict) or meta.get("scope") != "memory":
        out.issues.add("invalid_memory_sensor_scope")
        return out
    semantics, field_id = SOURCES.get(selected) or (None, None)
    if field_id and ("field" in meta and meta["field"] != field_id or "semantics" in meta and meta["semantics"] != semantics):
        out.issues.add("inconsistent_memory_sensor_metadata")
    if "timestamp_us" in meta:
        stamp = number(meta["timestamp_us"])
        if stamp is None or stamp < 0:
            out.issues.add("invalid_memory_sensor_timestamp")
        else:
            out.timestamp = stamp
            clock = meta.get("timestamp_clock")
            if clock is not None and clock != UNIX_US:
                out.issues.add("invalid_memory_sensor_timestamp_clock")
            q0, q1 = number(sample.get("query_realtime_start_s")), number(sample.get("query_realtime_end_s"))
            if clock == UNIX_US and q0 is not None and q1 is not None:
                if q1 < q0:
                    out.issues.add("invalid_memory_sensor_query_timestamps")
                else:
                    sensor_s = stamp / 1e6
                    out.age = max(0.0, q0 - sensor_s)
                    if out.age > maximum_age:
                        out.issues.add("stale_memory_sensor_timestamp")
                    if sensor_s > q1 + .001:
                        out.issues.add("future_memory_sensor_timestamp")
    if "latency_us" in meta and (number(meta["latency_us"]) is None or meta["latency_us"] < 0):
        out.issues.add("invalid_memory_sensor_latency")
    return out


# Window-level rules over the covering samples: (issue, predicate(covering, start, end, maximum_gap)).
WINDOW_RULES = (
    ("missing_memory_sensor_coverage", lambda c, a, b, gap: c[0]["t_s"] > a or c[-1]["t_s"] < b
     or any(number(s.get("memory_power_w")) is None for s in c)),
    ("negative_memory_sensor_power", lambda c, a, b, gap: any((v := number(s.get("memory_power_w"))) is not None and v < 0
                                                              for s in c)),
    ("memory_sensor_telemetry_gap", lambda c, a, b, gap: any(y["t_s"] - x["t_s"] > gap for x, y in zip(c, c[1:]))),
    ("unknown_memory_sensor_source", lambda c, a, b, gap: any(s.get("memory_power_source") not in SOURCES for s in c)),
    ("mixed_memory_sensor_sources", lambda c, a, b, gap: len({s.get("memory_power_source") for s in c}) != 1),
)


def phase_sensor(phase: Mapping | None, stats: Mapping, maximum_gap: float, energy: float | None) -> dict[str, Any]:
    """One window's memory-rail reading; ``energy`` is the kernel's trapezoid of memory_power_w over it."""
    result = empty()
    times, samples = _by_time(phase)
    start, end = number(stats.get("start_s")), number(stats.get("end_s"))
    reported = lambda group: any(s.get("memory_power_w") is not None for s in group)  # noqa: E731
    if start is None or end is None or end <= start:
        result.update(issues=["invalid_memory_sensor_window"], status="invalid" if reported(samples) else "unavailable")
        return result
    covering = _cover(times, samples, start, end)
    if not reported(covering):
        result["issues"] = ["memory_sensor_unavailable"]
        return result
    issues = {name for name, rule in WINDOW_RULES if rule(covering, start, end, maximum_gap)}
    sources = {s.get("memory_power_source") for s in covering}
    source = next(iter(sources)) if len(sources) == 1 and next(iter(sources)) in SOURCES else None
    maximum_age = max(MIN_STALE_AGE_S, maximum_gap)
    readings = [_inspect(s, maximum_age) for s in covering]
    for r in readings:
        issues |= r.issues
    stamps = [r.timestamp for r in readings if r.timestamp is not None]
    if any(b < a for a, b in zip(stamps, stamps[1:])):
        issues.add("memory_sensor_timestamp_regression")
    ages = [r.age for r in readings if r.age is not None]
    everywhere = len(ages) == len(covering)
    freshness = ("invalid" if ages and issues else "verified" if everywhere else "partial" if ages else "unverified")
    result.update(source=source, semantics=SOURCES[source][0] if source else None, freshness_maximum_age_s=maximum_age,
                  maximum_sensor_age_s=max(ages) if ages else None, freshness_status=freshness,
                  freshness_verified=everywhere and not issues)
    if energy is None:
        issues.add("missing_memory_sensor_coverage")
    result.update(issues=sorted(issues), status="invalid" if issues else "available", measurement_valid=not issues)
    if not issues:
        result.update(energy_j=energy, power_w=energy / (end - start))
    return result


# ---------------------------------------------------------------------------- trial record
def _idle_at(pre: Mapping, post: Mapping, active: Mapping, field: str) -> float | None:
    """Idle level interpolated at the active window's midpoint (analysis.py:210-216)."""
    a, b = number(pre.get(field)), number(post.get(field))
    t0, t1, t = number(pre.get("midpoint_s")), number(post.get("midpoint_s")), number(active.get("midpoint_s"))
    if any(v is None for v in (a, b, t0, t1, t)) or t1 <= t0 or not t0 <= t <= t1:
        return None
    return a + (b - a) * (t - t0) / (t1 - t0)


def _idle_baseline(sensor: dict, pre: dict, post: dict, phases: Mapping, maximum_idle_drift: float) -> list[str]:
    """The matched idle level under the measure window (into sensor["idle_power_w"]) and what prevents it."""
    problems = [f"{name}:{issue}" for name, window in (("idle_pre", pre), ("idle_post", post)) for issue in window["issues"]]
    if sensor["source"] is None or not pre["source"] == post["source"] == sensor["source"]:
        problems.append("idle_memory_sensor_source_mismatch")
    if problems:
        return problems
    idle = _idle_at(dict(phases["idle_pre"], memory_power_w=pre["power_w"]),
                    dict(phases["idle_post"], memory_power_w=post["power_w"]), phases["measure"], "memory_power_w")
    if idle is None:
        return ["missing_idle_memory_sensor_baseline"]
    sensor["idle_power_w"] = idle
    mean = max((pre["power_w"] + post["power_w"]) / 2, 1e-9)
    return ["memory_idle_baseline_drift"] if abs(pre["power_w"] - post["power_w"]) / mean > maximum_idle_drift else []


def trial_sensor(record: Mapping, result: Mapping, phases: Mapping, phase_records: Mapping,
                 maximum_gap: float, maximum_idle_drift: float) -> dict[str, Any] | None:
    """Memory-rail record of one HBM trial: the measure window's energy and power, per logical bit
    when the counts align, and above the matched idle level when both idle windows qualify."""
    if record.get("workload") != "hbm":
        return None
    window = {name: phase_sensor(phase_records.get(name), phases[name], maximum_gap,
                                 number(phases[name].get("memory_rail_energy_j")))
              for name in ("measure", "idle_pre", "idle_post")}
    sensor = window["measure"]
    bits = number(result.get("counted_measure_logical_bytes"))
    bits = bits * 8 if bits is not None and bits > 0 else None
    sensor["normalization_valid"] = bool(sensor["measurement_valid"] and result.get("valid")
                                         and result.get("count_energy_time_alignment_exact") is True and bits)
    if sensor["normalization_valid"]:
        sensor["pj_per_logical_bit"] = sensor["energy_j"] / bits * 1e12
    problems = _idle_baseline(sensor, window["idle_pre"], window["idle_post"], phases, maximum_idle_drift)
    if not sensor["measurement_valid"]:
        problems.append("invalid_treatment_memory_sensor")
    if result.get("operational_idle_increment_eligible") is not True:
        problems.append("unqualified_matched_idle_baseline")
    if not problems:
        sensor.update(incremental_power_w=sensor["power_w"] - sensor["idle_power_w"],
                      incremental_energy_j=sensor["energy_j"] - sensor["idle_power_w"] * result["duration_s"],
                      incremental_valid=True)
        if sensor["normalization_valid"]:
            sensor["incremental_pj_per_logical_bit"] = sensor["incremental_energy_j"] / bits * 1e12
    sensor["incremental_issues"] = sorted(set(problems))
    return sensor


def _population(sensor: Mapping, name: str) -> bool:
    """Whether a qualified repeat belongs to a field's population."""
    if name == "pj_per_logical_bit":
        return sensor["normalization_valid"]
    return sensor["incremental_valid"] if name.startswith("incremental_") else True


def bootstrap_columns(sensor: Mapping | None) -> list[float]:
    """One repeat's values of NUMERIC_FIELDS for the group bootstrap, NaN outside each field's population."""
    if not sensor or not sensor["measurement_valid"]:
        return [math.nan] * len(NUMERIC_FIELDS)
    values = [number(sensor[name]) if _population(sensor, name) else None for name in NUMERIC_FIELDS]
    return [math.nan if v is None else v for v in values]


# ---------------------------------------------------------------------------- group record
def _freshness(measured: list) -> tuple[bool, str]:
    verified = all(s["freshness_verified"] for s in measured)
    if verified:
        return True, "verified"
    return False, "partial" if any(s["freshness_status"] != "unverified" for s in measured) else "unverified"


def group_sensor(trials: list, workload: str, observed_trials: list | None,
                 medians: list, intervals: list) -> dict[str, Any] | None:
    """Repeat medians and intervals of the memory-rail fields of a group.

    ``medians``/``intervals`` hold, per NUMERIC_FIELDS entry, the median and
    the [lo, hi] interval the bootstrap kernel computed over
    ``bootstrap_columns`` of the group's valid repeats.
    """
    if workload != "hbm":
        return None
    result = empty()
    observed = trials if observed_trials is None else observed_trials
    sensors = [t["hbm_memory_power"] for t in trials]
    measured = [s for s in sensors if s["measurement_valid"]]
    board_invalid = sum(t.get("valid") is not True for t in observed)
    duplicates = len(observed) - len(trials) - board_invalid
    result.update(observed_repeats=len(observed), valid_repeats=len(measured),
                  normalized_repeats=sum(1 for s in measured if s["normalization_valid"]),
                  incremental_repeats=sum(1 for s in measured if s["incremental_valid"]),
                  board_invalid_repeats=board_invalid, duplicate_repeats_excluded=duplicates,
                  ci95=dict.fromkeys(NUMERIC_FIELDS))
    result["issues"] = (sorted({i for s in sensors for i in s["issues"]})
                        + (["board_invalid_repeats_excluded"] if board_invalid else [])
                        + (["duplicate_repeat_indices_excluded"] if duplicates else []))
    result["incremental_issues"] = sorted({i for s in sensors for i in s["incremental_issues"]})
    if len({s["source"] for s in measured}) > 1:
        result.update(status="invalid", issues=sorted(set(result["issues"]) | {"mixed_memory_sensor_sources_across_repeats"}))
        return result
    if not measured:
        every_board_invalid = bool(observed) and board_invalid == len(observed)
        result["status"] = ("invalid" if every_board_invalid or any(s["status"] == "invalid" for s in sensors)
                            else "unavailable")
        return result
    verified, freshness = _freshness(measured)
    ages = [s["maximum_sensor_age_s"] for s in measured if s["maximum_sensor_age_s"] is not None]
    result.update(status="available" if len(measured) == len(observed) else "partial",
                  source=measured[0]["source"], semantics=measured[0]["semantics"], measurement_valid=True,
                  normalization_valid=result["normalized_repeats"] > 0, incremental_valid=result["incremental_repeats"] > 0,
                  freshness_verified=verified, freshness_status=freshness,
                  maximum_sensor_age_s=max(ages) if ages else None,
                  freshness_maximum_age_s=min(s["freshness_maximum_age_s"] for s in measured))
    for k, name in enumerate(NUMERIC_FIELDS):
        result[name] = medians[k]
        result["ci95"][name] = intervals[k]
    return result


def host_median(values: list[float]) -> float | None:
    """statistics.median of the finite values (used where a group has no bootstrap columns)."""
    vals = [v for v in values if v is not None]
    return statistics.median(vals) if vals else None
