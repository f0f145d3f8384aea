"""HBM logical-bandwidth admission against the clock-specific interface ceiling.

A trial's sustained logical rate (the kernel-computed ``throughput_bytes_s``)
is compared with the DDR interface ceiling at the memory clock the trial ran
at: 2 x memory MHz x 1e6 x bus bits / 8, the clock being the median over
the trial's aligned measure window (the reference's hbm_bandwidth.py:42-125
defines the gate and the record).

The assessment is written as evidence plus findings.  ``_trial_evidence``
derives every fact once (bus width, window clock, MIG state, rate, ceiling,
fraction); each finding in the tables below is a named predicate over those
facts, of one of three kinds: a gap in the evidence (the trial cannot be
judged: ``inconclusive``), a failed gate (``fail``), or a warning.  One
function turns the fired findings into the record.
"""
from __future__ import annotations

import math
import statistics
from dataclasses import dataclass
from typing import Any, Callable, Mapping

DEFAULT_FRACTION = 0.80
FORMULA = "2 * memory_clock_mhz * 1e6 * memory_bus_width_bits / 8"
SCOPE = ("Sustained matching-window logical payload versus the clock-specific DDR interface ceiling; "
         "not simultaneous physical DRAM utilization or isolated memory energy. "
         "Observed-peak ratios and resource plateaus are diagnostics for HBM, not candidate gates.")
GROUP_AGGREGATION = ("Median of valid repeat logical bandwidth fractions; every valid repeat needs complete "
                     "bus/clock evidence. Above-interface logical rates are warnings, not physical-traffic contradictions.")
BELOW = "below_hbm_theoretical_bandwidth_fraction"
# Fields a group reports as the median over its valid repeats.
MEDIAN_FIELDS = ("theoretical_bytes_s", "sustained_logical_bytes_s", "fraction_of_theoretical",
                 "achieved_memory_clock_mhz", "memory_bus_width_bits")


def _finite(value) -> float | None:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
        return None
    return float(value)


def validate_fraction(value):
    value = _finite(value)
    if value is None or not 0 < value <= 1:
        raise ValueError("hbm_bandwidth_fraction must be finite and in (0, 1]")
    return value


def theoretical_bytes_s(memory_clock_mhz: float, bus_bits: float) -> float:
    return 2 * memory_clock_mhz * 1e6 * bus_bits / 8


@dataclass
class _Evidence:
    bus: float | None
    clock: float | None
    uuid_mismatch: bool
    mig: str                      # "off", "active" (unqualified) or "unknown"
    rate: float | None            # as reported (a non-positive rate is kept, and flagged)
    rate_ok: bool
    peak: float | None
    peak_invalid: bool
    cache_policy_ok: bool
    minimum: float

    @property
    def ratio(self) -> float | None:
        return self.rate / self.peak if self.rate is not None and self.peak and self.peak > 0 else None


@dataclass(frozen=True)
class Finding:
    name: str
    kind: str                     # "evidence" | "gate" | "warning"
    fires: Callable[[_Evidence], bool]


# In report order: the evidence a fraction needs, then the gates, then warnings.
TRIAL_FINDINGS = (
    Finding("missing_or_invalid_memory_bus_width_bits", "evidence", lambda e: e.bus is None),
    Finding("incomplete_measure_window_memory_clock_telemetry", "evidence", lambda e: e.clock is None),
    Finding("cuda_device_uuid_mismatch", "evidence", lambda e: e.uuid_mismatch),
    Finding("mig_memory_bus_mapping_unqualified", "evidence", lambda e: e.mig == "active"),
    Finding("unknown_mig_memory_bus_mapping", "evidence", lambda e: e.mig == "unknown"),
    Finding("missing_or_invalid_sustained_logical_bandwidth", "evidence", lambda e: not e.rate_ok),
    Finding("invalid_theoretical_bandwidth", "evidence", lambda e: e.peak_invalid),
    Finding("hbm_read_cache_policy_requires_cg", "gate", lambda e: not e.cache_policy_ok),
    Finding(BELOW, "gate", lambda e: e.ratio is not None and e.ratio < e.minimum),
    Finding("logical_rate_above_interface_ceiling_cache_reuse_or_count_review", "warning",
            lambda e: e.ratio is not None and e.ratio > 1 + 1e-9),
)


def _mig_state(record: Mapping) -> str:
    """'active' when MIG is on (or the device is a MIG instance), 'unknown' when the mode could
    not be read for a reason other than the device not supporting MIG, else 'off'."""
    device, cuda = record.get("device") or {}, record.get("cuda_device") or {}
    mode = device.get("mig_mode", cuda.get("mig_mode"))
    current = mode.get("current") if isinstance(mode, dict) else mode
    ids = (cuda.get("uuid"), device.get("uuid"), (record.get("config") or {}).get("gpu_uuid"))
    if (current in (1, True, "enabled", "Enabled") or (record.get("quality") or {}).get("mig_active") is True
            or any(str(u).startswith("MIG-") for u in ids)):
        return "active"
    if "mig_mode" in device:
        reported = device["mig_mode"]
        if reported is None or isinstance(reported, dict) and reported.get("current") is None:
            error = (device.get("errors") or {}).get("mig_mode") or {}
            if error.get("code") != 3 and error.get("type") != "NVMLError_NotSupported":
                return "unknown"
    return "off"


def _trial_evidence(record: Mapping, trial: Mapping, selected_samples, minimum: float) -> _Evidence:
    cuda = record.get("cuda_device") or {}
    bus = _finite(cuda.get("memory_bus_width_bits"))
    if bus is not None and (bus <= 0 or not bus.is_integer() or bus % 8):
        bus = None
    clocks = [_finite(s.get("memory_clock_mhz")) for s in selected_samples]
    clock = statistics.median(clocks) if clocks and all(c is not None and c > 0 for c in clocks) else None
    rate = _finite(trial.get("throughput_bytes_s"))
    peak = theoretical_bytes_s(clock, bus) if clock is not None and bus is not None else None
    peak_invalid = peak is not None and not math.isfinite(peak)
    contract = trial.get("experiment_contract") or {}
    return _Evidence(bus=bus, clock=clock,
                     uuid_mismatch=bool(cuda.get("uuid") and trial.get("gpu_uuid") and cuda["uuid"] != trial["gpu_uuid"]),
                     mig=_mig_state(record), rate=rate, rate_ok=rate is not None and rate > 0,
                     peak=None if peak_invalid else peak, peak_invalid=peak_invalid,
                     cache_policy_ok=not (contract.get("access", "read") == "read"
                                          and contract.get("read_cache_policy", "cg") != "cg"),
                     minimum=minimum)


def _status(eligible: bool, complete: bool) -> str:
    return "pass" if eligible else "inconclusive" if not complete else "fail"


def trial_bandwidth(record, trial, selected_samples, minimum_fraction=DEFAULT_FRACTION) -> dict[str, Any] | None:
    """The HBM bandwidth record of one trial (None for other workloads)."""
    minimum_fraction = validate_fraction(minimum_fraction)
    if trial.get("workload") != "hbm":
        return None
    e = _trial_evidence(record, trial, selected_samples, minimum_fraction)
    fired = [f for f in TRIAL_FINDINGS if f.fires(e)]
    reasons = [f.name for f in fired if f.kind != "warning"]
    complete = not any(f.kind == "evidence" for f in fired)
    return {"status": _status(not reasons, complete), "eligible": not reasons, "evidence_complete": complete,
            "minimum_fraction": minimum_fraction, "theoretical_bytes_s": e.peak, "sustained_logical_bytes_s": e.rate,
            "fraction_of_theoretical": e.ratio, "achieved_memory_clock_mhz": e.clock, "memory_bus_width_bits": e.bus,
            "clock_source": "matching_measure_window_memory_clock_mhz", "formula": FORMULA,
            "physical_dram_utilization_measured": False, "reasons": reasons,
            "warnings": [f.name for f in fired if f.kind == "warning"], "scope": SCOPE}


def group_bandwidth(valid_trials, workload, minimum_fraction=DEFAULT_FRACTION) -> dict[str, Any] | None:
    """The HBM bandwidth record of a group: medians over its valid repeats' trial records."""
    minimum_fraction = validate_fraction(minimum_fraction)
    if workload != "hbm":
        return None
    trials = list(valid_trials)
    present = [r for r in (t.get("hbm_bandwidth") for t in trials) if isinstance(r, dict)]
    every_repeat = bool(trials) and len(present) == len(trials)
    one_bus = len({r.get("memory_bus_width_bits") for r in present}) <= 1
    complete = every_repeat and one_bus and all(r.get("evidence_complete") is True for r in present)
    medians = {}
    for name in MEDIAN_FIELDS:
        values = [_finite(r.get(name)) for r in present]
        medians[name] = statistics.median(values) if complete and None not in values else None
    # The repeats' own reasons, except their individual fraction verdicts (the group decides on the median).
    reasons = {x for r in present for x in r.get("reasons", []) if x != BELOW}
    for name, missing in (("missing_valid_repeat_hbm_bandwidth_evidence", not every_repeat),
                          ("inconsistent_valid_repeat_memory_bus_width_bits", not one_bus),
                          (BELOW, medians["fraction_of_theoretical"] is not None
                           and medians["fraction_of_theoretical"] < minimum_fraction)):
        if missing:
            reasons.add(name)
    eligible = complete and medians["fraction_of_theoretical"] is not None and not reasons
    return {"status": _status(eligible, complete), "eligible": eligible, "evidence_complete": complete,
            "minimum_fraction": minimum_fraction, **medians,
            "clock_source": "matching_measure_window_memory_clock_mhz", "formula": FORMULA,
            "physical_dram_utilization_measured": False, "reasons": sorted(reasons),
            "warnings": sorted({x for r in present for x in r.get("warnings", [])}),
            "scope": SCOPE, "valid_repeats": len(trials), "evidence_repeats": len(present),
            "aggregation": GROUP_AGGREGATION}
