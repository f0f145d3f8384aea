"""HBM logical-bandwidth admission against the clock-specific interface ceiling.

Restates powermodeling/hbm_bandwidth.py (trial_bandwidth 42-91,
group_bandwidth 94-125): theory = 2 * memory MHz * 1e6 * bus bits / 8, the
measured memory clock being the median over the trial's aligned measure
window, and a trial qualifies at >= ``minimum_fraction`` of it.  The logical
rate is the kernel-computed ``throughput_bytes_s``.
"""
from __future__ import annotations

import math
import statistics

DEFAULT_FRACTION = 0.80
FORMULA = "2 * memory_clock_mhz * 1e6 * memory_bus_width_bits / 8"
SCOPE = ("Sustained matching-window logical payload versus the clock-specific DDR interface ceiling; "
         "not simultaneous physical DRAM utilization or isolated memory energy. "
         "Observed-peak ratios and resource plateaus are diagnostics for HBM, not candidate gates.")


def _number(value):
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        return None
    return float(value) if math.isfinite(value) else None


def validate_fraction(value):
    value = _number(value)
    if value is None or not 0 < value <= 1:
        raise ValueError("hbm_bandwidth_fraction must be finite and in (0, 1]")
    return value


def _mig_active(record) -> bool:
    device, cuda = record.get("device") or {}, record.get("cuda_device") or {}
    mode = device.get("mig_mode", cuda.get("mig_mode"))
    current = mode.get("current") if isinstance(mode, dict) else mode
    uuids = (cuda.get("uuid"), device.get("uuid"), (record.get("config") or {}).get("gpu_uuid"))
    return (current in (1, True, "enabled", "Enabled") or (record.get("quality") or {}).get("mig_active") is True
            or any(str(u).startswith("MIG-") for u in uuids))


def theoretical_bytes_s(memory_clock_mhz: float, bus_bits: float) -> float:
    return 2 * memory_clock_mhz * 1e6 * bus_bits / 8


def trial_bandwidth(record, trial, selected_samples, minimum_fraction=DEFAULT_FRACTION):
    minimum_fraction = validate_fraction(minimum_fraction)
    if trial.get("workload") != "hbm":
        return None
    reasons: list[str] = []
    cuda = record.get("cuda_device") or {}
    bus = _number(cuda.get("memory_bus_width_bits"))
    if bus is None or bus <= 0 or not bus.is_integer() or bus % 8:
        bus = None
        reasons.append("missing_or_invalid_memory_bus_width_bits")
    clocks = [_number(s.get("memory_clock_mhz")) for s in selected_samples]
    complete = bool(clocks) and all(c is not None and c > 0 for c in clocks)
    clock = statistics.median(clocks) if complete else None
    if not complete:
        reasons.append("incomplete_measure_window_memory_clock_telemetry")
    if cuda.get("uuid") and trial.get("gpu_uuid") and cuda["uuid"] != trial["gpu_uuid"]:
        reasons.append("cuda_device_uuid_mismatch")
    device = record.get("device") or {}
    if _mig_active(record):
        reasons.append("mig_memory_bus_mapping_unqualified")
    elif "mig_mode" in device and (device.get("mig_mode") is None or
                                   isinstance(device.get("mig_mode"), dict) and device["mig_mode"].get("current") is None):
        error = (device.get("errors") or {}).get("mig_mode") or {}
        if error.get("code") != 3 and error.get("type") != "NVMLError_NotSupported":
            reasons.append("unknown_mig_memory_bus_mapping")
    rate = _number(trial.get("throughput_bytes_s"))
    if rate is None or rate <= 0:
        reasons.append("missing_or_invalid_sustained_logical_bandwidth")
    peak = theoretical_bytes_s(clock, bus) if clock is not None and bus is not None else None
    if peak is not None and not math.isfinite(peak):
        peak = None
        reasons.append("invalid_theoretical_bandwidth")
    ratio = rate / peak if rate is not None and peak and peak > 0 else None
    complete_evidence = not reasons
    warnings: list[str] = []
    contract = trial.get("experiment_contract") or {}
    if contract.get("access", "read") == "read" and contract.get("read_cache_policy", "cg") != "cg":
        reasons.append("hbm_read_cache_policy_requires_cg")
    if ratio is not None and ratio > 1 + 1e-9:
        warnings.append("logical_rate_above_interface_ceiling_cache_reuse_or_count_review")
    if ratio is not None and ratio < minimum_fraction:
        reasons.append("below_hbm_theoretical_bandwidth_fraction")
    return {"status": "pass" if not reasons else "inconclusive" if not complete_evidence else "fail",
            "eligible": not reasons, "evidence_complete": complete_evidence, "minimum_fraction": minimum_fraction,
            "theoretical_bytes_s": peak, "sustained_logical_bytes_s": rate, "fraction_of_theoretical": ratio,
            "achieved_memory_clock_mhz": clock, "memory_bus_width_bits": bus,
            "clock_source": "matching_measure_window_memory_clock_mhz", "formula": FORMULA,
            "physical_dram_utilization_measured": False, "reasons": reasons, "warnings": warnings, "scope": SCOPE}


def group_bandwidth(valid_trials, workload, minimum_fraction=DEFAULT_FRACTION):
    minimum_fraction = validate_fraction(minimum_fraction)
    if workload != "hbm":
        return None
    trials = list(valid_trials)
    present = [r for r in (t.get("hbm_bandwidth") for t in trials) if isinstance(r, dict)]
    complete = bool(trials) and len(present) == len(trials) and all(r.get("evidence_complete") is True for r in present)
    reasons = sorted({x for r in present for x in r.get("reasons", []) if x != "below_hbm_theoretical_bandwidth_fraction"})
    warnings = sorted({x for r in present for x in r.get("warnings", [])})
    if len(present) != len(trials) or not trials:
        reasons.append("missing_valid_repeat_hbm_bandwidth_evidence")
    if len({r.get("memory_bus_width_bits") for r in present}) > 1:
        complete = False
        reasons.append("inconsistent_valid_repeat_memory_bus_width_bits")

    def median(name):
        values = [_number(r.get(name)) for r in present]
        return statistics.median(values) if complete and all(v is not None for v in values) else None

    ratio = median("fraction_of_theoretical")
    if ratio is not None and ratio < minimum_fraction:
        reasons.append("below_hbm_theoretical_bandwidth_fraction")
    eligible = complete and ratio is not None and not reasons
    return {"status": "pass" if eligible else "inconclusive" if not complete else "fail",
            "eligible": eligible, "evidence_complete": complete, "minimum_fraction": minimum_fraction,
            **{name: median(name) for name in ("theoretical_bytes_s", "sustained_logical_bytes_s",
                                               "fraction_of_theoretical", "achieved_memory_clock_mhz",
                                               "memory_bus_width_bits")},
            "clock_source": "matching_measure_window_memory_clock_mhz", "formula": FORMULA,
            "physical_dram_utilization_measured": False, "reasons": sorted(set(reasons)), "warnings": warnings,
            "scope": SCOPE, "valid_repeats": len(trials), "evidence_repeats": len(present),
            "aggregation": "Median of valid repeat logical bandwidth fractions; every valid repeat needs complete "
                           "bus/clock evidence. Above-interface logical rates are warnings, not physical-traffic contradictions."}
