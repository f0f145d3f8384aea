"""B200 analysis of sustained-power trials, with the reference's Python interface.

``analyze_trial``/``analyze_trials``/``summarize``/``median_ci`` take the same
arguments and return the same keys as powermodeling.analysis (analysis.py:597,
1400, 1096) for the numeric core of a trial and a group: phase integrals over
aligned completion epochs, idle-delta and paired-reference contrasts, pJ per
FLOP/bit/op, group medians and bootstrap intervals.  Every number comes from
libpmb200's kernels (pm_analyze_trials, pm_group_bootstrap); this module only
packs records, turns issue bits into the reference's strings and builds the
group keys whose sha256 prefix seeds each group's resampling.

Outside this module's scope, and absent from its dicts: Nsight Compute
evidence assessment (validation.py), memory-coalescing geometry, evaluation,
selections and optima (analysis.py:1122-1398), and measurement diagnostics.
``target_verified`` is therefore always False, as the reference reports for
a trial without profiler evidence.
"""
from __future__ import annotations

import gc
import hashlib
import json
import math
import statistics
from dataclasses import asdict, dataclass, replace
from typing import Any, Iterable, Mapping

import numpy as np

from . import _native as N
from . import contracts
from .pack import (MEMORY_WORKLOADS, NONLINEAR_WORKLOADS, ROW_WORKLOADS, SFU_WORKLOADS, TENSOR_WORKLOADS,
                   finite, pack_trials, phase_records, trials_struct)
from .memory_power import ALIASES as SENSOR_ALIASES
from .memory_power import NUMERIC_FIELDS as SENSOR_FIELDS
from .memory_power import bootstrap_columns as sensor_columns
from .memory_power import group_sensor, trial_sensor
from .profiles import ARCHITECTURES

ENERGY_WORKLOADS = TENSOR_WORKLOADS | MEMORY_WORKLOADS | SFU_WORKLOADS | NONLINEAR_WORKLOADS
DEFAULT_RESAMPLES = 1000

METRICS = ("board_power_w", "idle_power_w", "incremental_power_w", "throughput_ops_s", "throughput_bytes_s",
           "pj_per_op", "pj_per_logical_byte", "total_pj_per_op", "total_pj_per_logical_byte",
           "memory_rail_power_w", "memory_rail_incremental_power_w", "graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz",
           "temperature_c", "idle_fraction_of_measured_power", "idle_fraction_of_power_limit", "power_limit_utilization",
           "tensor_peak_tflops_at_achieved_clock", "tensor_utilization_vs_dense_clock_peak",
           "total_pj_per_flop", "total_pj_per_logical_bit",
           "operational_idle_increment_power_w", "operational_idle_increment_energy_j",
           "operational_idle_increment_pj_per_flop", "operational_idle_increment_pj_per_logical_bit",
           "paired_active_reference_power_w", "paired_active_reference_energy_j",
           "paired_active_reference_pj_per_flop", "paired_active_reference_pj_per_logical_bit",
           "throughput_elements_s", "throughput_rows_s", "total_pj_per_element", "total_pj_per_row",
           "operational_idle_increment_pj_per_element", "operational_idle_increment_pj_per_row",
           "paired_active_reference_pj_per_element", "paired_active_reference_pj_per_row",
           "throughput_sfu_instructions_s", "total_pj_per_instruction", "operational_idle_increment_pj_per_instruction",
           "paired_active_reference_pj_per_instruction", "sfu_reference_delta_pj_per_instruction", "sfu_reference_delta_power_w",
           "active_reference_duration_s", "active_reference_counted_loop_slots", "active_reference_loop_slots_s")
"""The reference's _METRICS tuple (analysis.py:1059-1074); libpmb200 writes its rows in this order."""

REPEAT_KEYS = {"repeat", "repeat_id", "repeat_index", "trial_id", "output_dir", "output_path"}


@dataclass(frozen=True)
class AnalysisPolicy:
    """Same fields, defaults and validation as the reference's (analysis.py:42-67)."""
    trim_s: float = 2.0
    idle_trim_s: float = 1.0
    min_measure_s: float = 5.0
    min_idle_s: float = 4.0
    min_samples: int = 4
    max_sample_gap_s: float = 2.5
    clock_tolerance_fraction: float = 0.03
    max_clock_drift_fraction: float = 0.03
    max_temperature_drift_c: float = 5.0
    max_idle_drift_fraction: float = 0.10
    counter_disagreement_fraction: float = 0.10
    near_optimum_fraction: float = 0.05
    min_geometries: int = 2

    def __post_init__(self):
        for name, value in asdict(self).items():
            if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value) or value < 0:
                raise ValueError(f"Analysis policy {name} must be finite and nonnegative")
        if type(self.min_samples) is not int or self.min_samples < 2:
            raise ValueError("min_samples must be an integer >=2")
        if type(self.min_geometries) is not int or self.min_geometries < 2:
            raise ValueError("min_geometries must be an integer >=2; one geometry cannot qualify utilization")
        if self.min_measure_s <= 0 or self.min_idle_s <= 0 or self.max_sample_gap_s <= 0:
            raise ValueError("Measurement, idle and sample-gap durations must be positive")

    def native(self) -> N.Policy:
        return N.Policy(self.trim_s, self.idle_trim_s, self.min_measure_s, self.min_idle_s, self.min_samples,
                        self.max_sample_gap_s, self.clock_tolerance_fraction, self.max_clock_drift_fraction,
                        self.max_temperature_drift_c, self.max_idle_drift_fraction, self.counter_disagreement_fraction)


def _policy(policy) -> AnalysisPolicy:
    return policy if isinstance(policy, AnalysisPolicy) else AnalysisPolicy(**(policy or {}))


def _none(x) -> float | None:
    """NaN (the ABI's None) -> None; Python floats otherwise."""
    x = float(x)
    return None if math.isnan(x) else x


def _py_rows(values: np.ndarray, width: int) -> list[list]:
    """A result array as rows of Python floats, NaN (the ABI's None) as None: _none on every element at once."""
    obj = values.astype(object)
    obj[np.isnan(values)] = None
    return obj.reshape(-1, width).tolist() if width else []


# --- issue strings for each bit word ----------------------------------------
_PHASE_ISSUES = ("missing_phase", "invalid_phase_window", "short_plateau", "too_few_samples", "telemetry_gap",
                 "negative_power", "missing_power_coverage", "energy_counter_disagreement")
_EPOCH_ISSUES = ("invalid_measure_epochs_phase_window", "invalid_measure_epoch_boundaries",
                 "invalid_measure_epoch_count:operations", "invalid_measure_epoch_count:logical_bytes",
                 "overlapping_measure_epochs", "insufficient_complete_measure_epochs",
                 "measure_epoch_total_disagreement:operations", "measure_epoch_total_disagreement:logical_bytes",
                 "invalid_measure_epoch")
_CLOCKS = ("graphics_clock_mhz", "memory_clock_mhz", "sm_clock_mhz")


def _treatment_strings() -> list[str | None]:
    out = [f"{i}:measure" for i in _PHASE_ISSUES] + list(_EPOCH_ISSUES)
    out += [f"missing_clock_telemetry:{c}" for c in _CLOCKS] + [f"clock_mismatch:{c}" for c in _CLOCKS]
    out += [f"clock_drift:{c}" for c in _CLOCKS]
    out += ["temperature_drift", "missing_temperature_telemetry", "missing_throttling_telemetry", "active_throttling",
            "missing_process_inventory:compute_processes", "missing_process_inventory:graphics_processes",
            "missing_measurement_pid", "other_gpu_processes", "mps_active", "host_device_duration_disagreement",
            "missing_benchmark_duration", "missing_operation_count", "missing_logical_byte_count",
            "nonlinear_requires_matching_work_energy_epochs", "sfu_requires_matching_work_energy_epochs"]
    return out


def _baseline_strings() -> list[str]:
    out = [f"{i}:idle_pre" for i in _PHASE_ISSUES] + [f"{i}:idle_post" for i in _PHASE_ISSUES]
    out += ["idle_baseline_drift", "missing_idle_baseline", "negative_incremental_energy",
            "missing_process_inventory:compute_processes", "missing_process_inventory:graphics_processes",
            "missing_measurement_pid", "baseline_other_gpu_processes", "mps_active",
            "idle_state_mismatch_or_unverified:idle_pre:enforced_power_limit_w",
            "idle_state_mismatch_or_unverified:idle_pre:pstate",
            "idle_state_mismatch_or_unverified:idle_post:enforced_power_limit_w",
            "idle_state_mismatch_or_unverified:idle_post:pstate"]
    return out


def _paired_strings() -> list[str]:
    out = [f"{i}:active_reference" for i in _PHASE_ISSUES] + list(_EPOCH_ISSUES)
    out += ["reference_work_energy_window_unverified"]
    out += [f"paired_state_mismatch:{c}" for c in _CLOCKS] + ["paired_state_mismatch:temperature_c"]
    out += ["reference_throttle_unverified_or_active", "reference_process_inventory_unverified:compute_processes",
            "reference_process_inventory_unverified:graphics_processes", "reference_foreign_gpu_process",
            "paired_power_cap_unverified", "paired_power_cap_changed",
            "paired_state_mismatch:enforced_power_limit_w", "paired_state_mismatch:pstate",
            "paired_power_unavailable",
            "nonpositive_paired_contrast; signed observation retained but cannot minimize an energy objective",
            "missing_paired_active_reference_phase"]
    return out


_WARNINGS = ("energy_counter_reset:idle_pre", "energy_counter_reset:measure", "energy_counter_reset:idle_post",
             "energy_counter_reset:active_control", "uncontrolled_clock:graphics_clock_mhz",
             "uncontrolled_clock:memory_clock_mhz",
             "throughput_time_alignment_unverified; energy per work is a rate estimate assuming stationary throughput",
             "memory_rail_source_changed; rail incremental energy withheld",
             "tensor_peak_uses_graphics_clock_proxy; measured SM clock unavailable",
             "tensor_theoretical_peak_unavailable",
             "idle_active_pstate_or_enforced_cap_mismatch_or_unavailable; operational idle contrast is withheld from optimization",
             "idle_active_power_cap_mismatch_or_unavailable; idle contrast is withheld from optimization",
             "idle_active_clock_mismatch_or_unavailable; incremental power includes activation and frequency-state differences",
             "idle_active_temperature_mismatch_or_unavailable; leakage/thermal drift can confound subtraction")

_WORD_STRINGS = None


def _word_strings():
    global _WORD_STRINGS
    if _WORD_STRINGS is None:
        words = (_treatment_strings(), _baseline_strings(), _paired_strings(), list(_WARNINGS))
        counts = [N.layout(name) for name in ("PM_IT_COUNT", "PM_IB_COUNT", "PM_IP_COUNT", "PM_W_COUNT")]
        for strings, count in zip(words, counts):
            if len(strings) != count:
                raise N.NativeError(f"issue table mismatch: {len(strings)} strings for {count} bits")
        _WORD_STRINGS = words
    return _WORD_STRINGS


def _bits(word: int, strings) -> list[str]:
    out = []
    while word:
        low = word & -word
        out.append(strings[low.bit_length() - 1])
        word ^= low
    return out


# --- record-level (host) checks -------------------------------------------------
def _host_treatment_issues(record, bench, config, device, epoch_status) -> list[str]:
    """analyze_trial's checks on record metadata alone (analysis.py:620-629, 666-697, 753-757)."""
    issues = []
    if epoch_status == N.EP_INVALID_LIST:
        issues.append("invalid_measure_epochs")
    if not record.get("trial_id"):
        issues.append("missing_trial_id")
    quality = record.get("quality") or {}
    if quality.get("valid") is False:
        issues.append("runner_quality_invalid")
    for key in ("interference_detected", "mig_active", "mps_active", "unsafe_short_duration"):
        if quality.get(key) or config.get(key):
            issues.append(key)
    if quality.get("other_compute_processes", record.get("other_compute_processes")):
        issues.append("other_compute_processes")
    mig_mode = device.get("mig_mode") or {}
    if isinstance(mig_mode, dict) and mig_mode.get("current"):
        issues.append("mig_active")
    if (record.get("provenance") or {}).get("mps_environment"):
        issues.append("mps_environment")
    if record.get("status") != "complete" or bench.get("error"):
        issues.append("benchmark_failed")
    sanity = bench.get("sanity") or {}
    sanity_map = type(sanity) is dict or isinstance(sanity, Mapping)
    if sanity_map and sanity.get("finite_output_sample") is False:
        issues.append("benchmark_output_sanity_failed")
    read_validation = bench.get("memory_read_validation") or {}
    if ((sanity_map and sanity.get("memory_read_sample_matches_reference") is False)
            or ((type(read_validation) is dict or isinstance(read_validation, Mapping)) and
                (read_validation.get("status") == "fail" or (finite(read_validation.get("mismatched_values")) or 0) > 0))):
        issues.append("memory_read_reference_mismatch")
    workload = record.get("workload")
    issues.extend(contracts.nonlinear_count_issues(bench, workload))
    issues.extend(contracts.memory_count_issues(bench, workload))
    issues.extend(contracts.sfu_count_issues(bench, workload))
    return issues


def _host_paired_issues(record, phases, epoch_status) -> list[str]:
    """_paired_reference_contrast's checks on record metadata (analysis.py:310-333, 370-371)."""
    protocol = record.get("treatment_protocol") or (record.get("benchmark") or {}).get("treatment_protocol") or {}
    reference = record.get("active_reference") or {}
    reference_phase = phases.get("active_reference")
    if not reference_phase:
        return []
    sfu = record.get("workload") in SFU_WORKLOADS
    issues = []
    if epoch_status == N.EP_INVALID_LIST:
        issues.append("invalid_measure_epochs")
    for name in ("same_process", "same_allocations", "same_clock_policy", "launch_geometry_matched"):
        if protocol.get(name) is not True:
            issues.append("paired_protocol_unverified:" + name)
    if (protocol.get("kind") != "paired_active_reference"
            or protocol.get("reference_kind") != (contracts.SFU_REFERENCE_KIND if sfu else "issue_loop")
            or protocol.get("reference_workload") != "control"):
        issues.append("paired_reference_definition_unverified")
    order = protocol.get("order")
    if order not in ("AB", "BA"):
        issues.append("paired_protocol_order_unverified")
    measure = phases.get("measure") or {}
    if order == "AB" and (finite(reference_phase.get("end_s")) or 0) > (finite(measure.get("start_s")) or 0):
        issues.append("paired_arm_order_or_overlap_invalid")
    if order == "BA" and (finite(measure.get("end_s")) or 0) > (finite(reference_phase.get("start_s")) or 0):
        issues.append("paired_arm_order_or_overlap_invalid")
    treatment = record.get("benchmark") or {}
    for name in ("blocks", "threads", "batch_launches", "iterations_per_launch"):
        if reference.get(name) is None or treatment.get(name) is None or reference[name] != treatment[name]:
            issues.append("paired_geometry_mismatch:" + name)
    if sfu:
        issues.extend(contracts.sfu_count_issues(reference, record.get("workload"), reference=True))
        for name in ("sfu_lanes", "sfu_chains", "sfu_primitive", "sfu_input_policy", "grid_mode",
                     "math_implementation", "sfu_ptx_opcode"):
            if reference.get(name) != treatment.get(name):
                issues.append("paired_sfu_contract_mismatch:" + name)
    if (reference.get("sanity") or {}).get("requested_sm_coverage_complete") is not True:
        issues.append("reference_sm_coverage_unverified")
    return issues


def _experiment_contract(workload, benchmark, config):
    """evaluation.experiment_contract (evaluation.py:32-58): part of the group key."""
    def get(key, default=None):
        return benchmark.get(key, config.get(key, default))
    if workload in MEMORY_WORKLOADS or workload == "l2_latency":
        size = get("working_set_bytes")
        if workload == "l1":
            blocks = get("blocks")
            size = get("l1_bytes_per_block", size / blocks if finite(size) is not None and finite(blocks) and blocks > 0 else None)
        contract = {"access": get("access", "read"),
                    "kernel_implementation_version": get("kernel_implementation_version"),
                    "read_cache_policy": get("read_cache_policy", "ca" if workload == "l1" else "cg"),
                    "memory_read_index_math": get("memory_read_index_math", "uint64"),
                    "memory_accesses_per_thread_iteration": get("memory_accesses_per_thread_iteration"),
                    ("l1_bytes_per_block" if workload == "l1" else "working_set_bytes"): size,
                    "stride_elements": get("stride_elements", 1)}
        if workload == "l2_latency":
            contract.update(blocks=get("blocks"), threads=get("threads"),
                            iterations_per_launch=get("iterations_per_launch", config.get("iterations")),
                            sm_filter_size=len(config.get("sm_ids") or []))
        else:
            contract.update(offset_bytes=get("offset_bytes", 0), sm_ids=config.get("sm_ids", []))
        return contract
    if workload in NONLINEAR_WORKLOADS:
        return {key: get(key) for key in ("working_set_bytes", "row_width", "input_precision", "math_implementation",
                                          "rms_epsilon", "affine_gamma", "nonlinear_input_distribution",
                                          "input_elements", "grid_mode", "kernel_implementation_version",
                                          "block_completion_count_source")}
    if workload in SFU_WORKLOADS:
        return {key: get(key) for key in contracts.SFU_CONTRACT_FIELDS}
    return ({"definition": "dense FP16 input / FP32 accumulation", "implementation": workload}
            if workload in TENSOR_WORKLOADS else {"definition": "active integer issue control"})


# --- result assembly -------------------------------------------------------------
class _Views:
    def __init__(self, n):
        self.PO = N.layout("PM_PO_COUNT")
        self.TO = N.layout("PM_TO_COUNT")
        self.phase_out = np.empty(n * N.PM_PHASES * self.PO)
        self.phase_flags = np.empty(n * N.PM_PHASES, dtype=np.uint32)
        self.trial_out = np.empty(n * self.TO)
        self.issue_bits = np.empty(n * 4, dtype=np.uint64)
        self.metrics = np.empty(n * len(METRICS))
        self.valid = np.empty(n, dtype=np.uint8)
        self.windows = None          # per slot (lo, hi) or None, read from phase_out once it is filled

    def struct(self) -> N.TrialResults:
        r = N.TrialResults()
        for name in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid"):
            setattr(r, name, getattr(self, name).ctypes.data)
        return r


_PO_NAMES = None


def _po_names():
    global _PO_NAMES
    if _PO_NAMES is None:
        names = {}
        for key in ("START_S", "END_S", "DURATION_S", "MIDPOINT_S", "SAMPLES", "GAP_MEDIAN_S", "GAP_MAX_S", "ENERGY_J",
                    "INTEGRATED_POWER_W", "POWER_W", "MEMORY_ENERGY_J", "MEMORY_POWER_W", "COUNTER_J", "DISAGREEMENT",
                    "DISTINCT_POWER", "CHANGE_MEDIAN_S"):
            names[key] = N.layout("PM_PO_" + key)
        for prefix, field in (("GFX", "graphics_clock_mhz"), ("SM", "sm_clock_mhz"), ("MEM", "memory_clock_mhz"),
                              ("TEMP", "temperature_c")):
            names[field] = tuple(N.layout(f"PM_PO_{prefix}_{s}") for s in ("MED", "MIN", "MAX"))
        _PO_NAMES = names
    return _PO_NAMES


_PF = None


def _pf_bits():
    """Phase flag bit positions: (missing, invalid window, counter reset, [(bit, issue) in report order])."""
    global _PF
    if _PF is None:
        issues = (("SHORT_PLATEAU", "short_plateau"), ("TOO_FEW_SAMPLES", "too_few_samples"),
                  ("TELEMETRY_GAP", "telemetry_gap"), ("NEGATIVE_POWER", "negative_power"),
                  ("MISSING_POWER_COVERAGE", "missing_power_coverage"), ("COUNTER_DISAGREEMENT", "energy_counter_disagreement"))
        _PF = (N.layout("PM_PF_MISSING"), N.layout("PM_PF_INVALID_WINDOW"), N.layout("PM_PF_COUNTER_RESET"),
               tuple((N.layout("PM_PF_" + key), text) for key, text in issues))
    return _PF


_CADENCE_NOTE = "Changes are not proof of sensor refresh cadence; unchanged values may be steady power."


def _phase_dict(name: str, po: np.ndarray, flags: int, policy: AnalysisPolicy, pv: list | None = None) -> dict:
    """The reference's _phase_stats dict without its private _selected list.

    ``pv``: the same phase row as Python values with None for NaN (``_py_rows``); derived from ``po`` when absent."""
    L = _po_names()
    missing, invalid, reset, issue_bits = _pf_bits()
    out: dict[str, Any] = {"name": name, "issues": [], "warnings": []}
    if flags >> missing & 1:
        out["issues"].append(f"missing_phase:{name}")
        return out
    if flags >> invalid & 1:
        out["issues"].append(f"invalid_phase_window:{name}")
        return out
    if pv is None:
        pv = _py_rows(np.asarray(po, dtype=np.float64), len(po))[0]
    samples = int(po[L["SAMPLES"]])
    out.update(start_s=pv[L["START_S"]], end_s=pv[L["END_S"]], duration_s=pv[L["DURATION_S"]],
               midpoint_s=pv[L["MIDPOINT_S"]], samples=samples,
               sample_interval_median_s=pv[L["GAP_MEDIAN_S"]], max_sample_gap_s=pv[L["GAP_MAX_S"]])
    for bit, text in issue_bits:
        if flags >> bit & 1:
            out["issues"].append(f"{text}:{name}")
    out["integrated_power_energy_j"] = pv[L["ENERGY_J"]]
    out["integrated_power_w"] = pv[L["INTEGRATED_POWER_W"]]
    out["power_w"] = pv[L["POWER_W"]]
    out["memory_rail_energy_j"] = pv[L["MEMORY_ENERGY_J"]]
    out["memory_power_w"] = pv[L["MEMORY_POWER_W"]]
    if flags >> reset & 1:
        out["warnings"].append(f"energy_counter_reset:{name}")
    out["energy_counter_j"] = pv[L["COUNTER_J"]]
    disagreement = pv[L["DISAGREEMENT"]]
    if disagreement is not None:
        out["counter_power_disagreement_fraction"] = disagreement
    out["distinct_power_values"] = int(po[L["DISTINCT_POWER"]])
    out["observed_power_change_interval_median_s"] = pv[L["CHANGE_MEDIAN_S"]]
    out["power_update_cadence_note"] = _CADENCE_NOTE
    for field in ("graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz", "temperature_c"):
        med, lo, hi = L[field]
        out[field] = pv[med]
        out[f"{field}_min"] = pv[lo]
        out[f"{field}_max"] = pv[hi]
    return out


def _phase_index() -> tuple:
    """Phase-row positions in the order _recordnative.phase_dicts takes them."""
    L = _po_names()
    scalars = ("START_S", "END_S", "DURATION_S", "MIDPOINT_S", "SAMPLES", "GAP_MEDIAN_S", "GAP_MAX_S", "ENERGY_J",
               "INTEGRATED_POWER_W", "POWER_W", "MEMORY_ENERGY_J", "MEMORY_POWER_W", "COUNTER_J", "DISAGREEMENT",
               "DISTINCT_POWER", "CHANGE_MEDIAN_S")
    clocks = ("graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz", "temperature_c")
    return tuple(L[k] for k in scalars) + tuple(i for field in clocks for i in L[field])


def _phase_dicts(views) -> list[dict]:
    """_phase_dict of every (trial, phase) slot of a result batch, built natively in one call."""
    from .trial_report import _record_native
    missing, invalid, reset, issue_bits = _pf_bits()
    return _record_native().phase_dicts(views.phase_out, views.phase_flags, views.PO, tuple(N.PHASE_NAMES),
                                        _phase_index(), (missing, invalid, reset), issue_bits, _CADENCE_NOTE)


def _gpu_uuid(record):
    config = dict(record.get("config") or {})
    device = record.get("device") or {}
    return config.get("gpu_uuid") or device.get("uuid") or record.get("gpu_uuid")


def _treatment_design_stratum(record, benchmark):
    protocol = record.get("treatment_protocol") or benchmark.get("treatment_protocol") or {}
    return {"kind": protocol.get("kind", "unspecified_legacy_protocol"),
            "reference_kind": protocol.get("reference_kind"),
            "paired_reference_context_allocated": benchmark.get("paired_reference_context_allocated",
                                                                protocol.get("paired_reference_context_allocated"))}


def prepare(records: list) -> tuple:
    """Record-level checks and the packed batch: (Packed, host issues, host paired issues)."""
    host_issues, host_paired, host_flags = [], [], []
    for record in records:
        bench = record.get("benchmark") or record.get("result") or {}
        config = dict(record.get("config") or {})
        device = record.get("device") or {}
        phases = phase_records(record)
        source = bench.get("measure_epochs", bench.get("work_epochs"))
        status = N.EP_NONE if source is None else (N.EP_INVALID_LIST if not isinstance(source, list) or not source else N.EP_OK)
        ref = record.get("active_reference") or {}
        rsource = ref.get("measure_epochs", ref.get("work_epochs"))
        rstatus = N.EP_NONE if rsource is None else (N.EP_INVALID_LIST if not isinstance(rsource, list) or not rsource else N.EP_OK)
        hi = _host_treatment_issues(record, bench, config, device, status)
        hp = _host_paired_issues(record, phases, rstatus)
        host_issues.append(hi)
        host_paired.append(hp)
        flags = (N.T_HOST_ISSUES if hi else 0) | (N.T_HOST_PAIRED if hp else 0)
        workload = record.get("workload")
        if workload in SFU_WORKLOADS and not contracts.sfu_count_issues(bench, workload):
            flags |= N.T_SFU_CONTRACT_OK
        if workload in NONLINEAR_WORKLOADS and not contracts.nonlinear_count_issues(bench, workload):
            flags |= N.T_NONLINEAR_OK
        host_flags.append(flags)
    return pack_trials(records, host_flags, ARCHITECTURES), host_issues, host_paired


def analyze_trials(records: Iterable[Mapping[str, Any]], policy: AnalysisPolicy | Mapping[str, Any] | None = None,
                   hbm_bandwidth_fraction: float = 0.80, _metrics_out: list | None = None) -> list[dict[str, Any]]:
    """analyze_trial over a batch, in one kernel launch."""
    from .hbm import trial_bandwidth, validate_fraction
    from .trial_report import complete_trial
    hbm_bandwidth_fraction = validate_fraction(hbm_bandwidth_fraction)
    policy = _policy(policy)
    records = list(records)
    if not records:
        return []
    words = _word_strings()
    packed, host_issues, host_paired = prepare(records)
    trials = trials_struct(packed)
    views = _Views(len(records))
    results = views.struct()
    N.check(N.library().pm_analyze_trials(trials, policy.native(), results), "pm_analyze_trials")
    if _metrics_out is not None:
        _metrics_out.append((views.metrics.reshape(len(records), len(METRICS)).copy(), views.valid.copy()))
    TO = {name: N.layout("PM_TO_" + name) for name in _TO_NAMES}
    to_rows = _py_rows(views.trial_out, views.TO)
    # the same rows as plain floats (NaN kept: flags are read with bool()), and the issue words as ints
    to_raw = views.trial_out.reshape(-1, views.TO).tolist()
    issue_rows = views.issue_bits.reshape(-1, 4).tolist()
    all_phases = _phase_dicts(views)
    policy_dict = asdict(policy)
    sel_lo, sel_hi = N.layout("PM_PO_SEL_LO"), N.layout("PM_PO_SEL_HI")
    out = []
    for i, record in enumerate(records):
        bench = record.get("benchmark") or record.get("result") or {}
        config = dict(record.get("config") or {})
        device = record.get("device") or {}
        phases_rec = phase_records(record)
        to = to_raw[i]
        to_py = to_rows[i]
        g = lambda name: to_py[TO[name]]  # noqa: E731
        ib = issue_rows[i]
        issues = host_issues[i] + _bits(ib[0], words[0])
        baseline_issues = _bits(ib[1], words[1])
        paired_issues = host_paired[i] + _bits(ib[2], words[2])
        warnings = _bits(ib[3], words[3])
        phase_dicts = dict(zip(N.PHASE_NAMES, all_phases[i * N.PM_PHASES:(i + 1) * N.PM_PHASES]))
        other_pids = set()
        measure_slot = i * N.PM_PHASES + 1
        mpo = views.phase_out[measure_slot * views.PO:(measure_slot + 1) * views.PO]
        lo, hi_ = mpo[sel_lo], mpo[sel_hi]
        if not math.isnan(lo):
            for index, pids in packed.foreign_pids[measure_slot]:
                if lo <= index < hi_:
                    other_pids.update(pids)
        workload = record.get("workload")
        duration = g("DURATION_S")
        power_limit = g("POWER_LIMIT_W")
        result: dict[str, Any] = {
            "trial_id": record.get("trial_id"), "condition_id": record.get("condition_id"), "workload": workload,
            "gpu_uuid": _gpu_uuid(record), "experiment_role": record.get("experiment_role", "legacy_unspecified"),
            "experiment_contract": _experiment_contract(workload, bench, config),
            "repeat_index": record.get("repeat", config.get("repeat", config.get("repeat_index"))),
            "gpu_name": device.get("name", record.get("gpu_name")), "config": config,
            "valid": not issues, "issues": sorted(set(issues)), "warnings": sorted(set(warnings)),
            "baseline_valid": not baseline_issues, "baseline_issues": sorted(set(baseline_issues)),
            "target_verified": False,
            "benchmark_sha256": (record.get("provenance") or {}).get("benchmark_sha256"),
            "treatment_design_stratum": _treatment_design_stratum(record, bench),
            "resource_geometry": {f: bench.get(f, config.get(f)) for f in (
                ("gemm_m", "gemm_n", "gemm_k") if workload == "gemm" else
                ("blocks", "threads", "tensor_accumulators") if workload in TENSOR_WORKLOADS else
                ("blocks", "threads", "sfu_chains") if workload in SFU_WORKLOADS else ("blocks", "threads"))},
            "sfu_contract": {f: bench.get(f) for f in contracts.SFU_CONTRACT_FIELDS} if workload in SFU_WORKLOADS else None,
            "nonlinear_contract": {f: bench.get(f) for f in (
                "row_width", "working_set_bytes", "input_elements", "grid_mode", "input_precision", "math_implementation",
                "kernel_implementation_version", "block_completion_count_source", "rms_epsilon", "affine_gamma",
                "nonlinear_input_distribution")} if workload in NONLINEAR_WORKLOADS else None,
            "measurement_stratum": {"ecc_mode": device.get("ecc_mode"), "mig_mode": device.get("mig_mode"),
                                    "driver_version": device.get("driver_version"), "nvml_version": device.get("nvml_version"),
                                    "runtime_versions": {k: (record.get("cuda_device") or {}).get(k) for k in (
                                        "cuda_runtime_version", "cuda_driver_version", "cuda_compile_version", "cublas_version")},
                                    "power_limit_w": power_limit,
                                    "power_scope": (record.get("telemetry") or {}).get("power_scope", device.get("power_scope_note")),
                                    "power_usage_semantics": device.get("power_usage_semantics"),
                                    "kernel_implementation_version": bench.get("kernel_implementation_version"),
                                    "block_completion_count_source": bench.get("block_completion_count_source"),
                                    "memory_accesses_per_thread_iteration": bench.get("memory_accesses_per_thread_iteration")},
            "kernel_implementation_version": bench.get("kernel_implementation_version"),
            "duration_s": duration, "benchmark_duration_s": g("BENCH_MEASURED_DURATION_S"),
            "benchmark_device_duration_s": g("BENCH_DEVICE_DURATION_S"),
            "count_energy_time_alignment_exact": bool(to[TO["EXACT"]]),
            "counted_measure_operations": g("COUNTED_OPS"), "counted_measure_logical_bytes": g("COUNTED_BYTES"),
            "complete_measure_epochs": int(to[TO["EPOCHS"]]),
            "energy_per_work_kind": "counted matching-window energy per work" if to[TO["EXACT"]] else "stationary whole-run-rate estimate",
            "diagnostic_only": workload not in ENERGY_WORKLOADS,
            "clock_comparison_controlled": all((finite(config.get(f)) or 0) > 0 for f in ("graphics_clock_mhz", "memory_clock_mhz")),
            "throughput_ops_s": g("OPS_RATE"), "throughput_bytes_s": g("BYTE_RATE"),
            "device_event_throughput_ops_s": g("DEVICE_OPS_RATE"), "device_event_throughput_bytes_s": g("DEVICE_BYTE_RATE"),
            "tensor_peak_tflops_at_achieved_clock": g("TENSOR_PEAK_TFLOPS"),
            "tensor_peak_clock_source": (("sm_clock_mhz" if to[TO["PEAK_CLOCK_IS_SM"]] else "graphics_clock_mhz")
                                         if g("TENSOR_PEAK_TFLOPS") is not None else None),
            "tensor_utilization_vs_dense_clock_peak": g("TENSOR_UTILIZATION"),
            "board_power_w": g("BOARD_POWER_W"), "idle_power_w": g("IDLE_POWER_W"), "incremental_power_w": g("INCREMENTAL_POWER_W"),
            "operational_idle_increment_power_w": g("INCREMENTAL_POWER_W"),
            "operational_idle_increment_energy_j": g("INCREMENTAL_ENERGY_J"),
            "operational_idle_increment_eligible": bool(to[TO["IDLE_INC_ELIGIBLE"]]) and not issues,
            "total_energy_j": g("TOTAL_ENERGY_J"), "idle_energy_j": g("IDLE_ENERGY_J"), "incremental_energy_j": g("INCREMENTAL_ENERGY_J"),
            "integrated_power_energy_j": phase_dicts["measure"].get("integrated_power_energy_j"),
            "energy_counter_j": phase_dicts["measure"].get("energy_counter_j"),
            "energy_source": "power_trapezoid" if to[TO["ENERGY_SOURCE_TRAPEZOID"]] else "energy_counter_delta",
            "pj_per_op": g("PJ_PER_OP"), "pj_per_logical_byte": g("PJ_PER_LOGICAL_BYTE"),
            "total_pj_per_op": g("TOTAL_PJ_PER_OP"), "total_pj_per_logical_byte": g("TOTAL_PJ_PER_LOGICAL_BYTE"),
            "memory_rail_power_w": phase_dicts["measure"].get("memory_power_w"), "memory_rail_idle_power_w": g("IDLE_MEMORY_POWER_W"),
            "memory_rail_energy_j": g("RAIL_ENERGY_J"), "memory_rail_incremental_energy_j": g("RAIL_INCREMENTAL_J"),
            "memory_rail_incremental_power_w": g("RAIL_INCREMENTAL_W"),
            "graphics_clock_mhz": phase_dicts["measure"].get("graphics_clock_mhz"),
            "sm_clock_mhz": phase_dicts["measure"].get("sm_clock_mhz"),
            "memory_clock_mhz": phase_dicts["measure"].get("memory_clock_mhz"),
            "temperature_c": phase_dicts["measure"].get("temperature_c"),
            "throttle_reasons_mask": int(to[TO["THROTTLE_MASK"]]) if not math.isnan(to[TO["THROTTLE_MASK"]]) else 0,
            "other_gpu_process_pids": sorted(other_pids),
            "power_limit_w": power_limit,
            "idle_fraction_of_measured_power": g("IDLE_FRAC_MEASURED"), "idle_fraction_of_power_limit": g("IDLE_FRAC_LIMIT"),
            "power_limit_utilization": g("LIMIT_UTILIZATION"),
            "baseline_clock_matched": bool(to[TO["BASE_CLOCK_MATCHED"]]),
            "baseline_temperature_matched": bool(to[TO["BASE_TEMP_MATCHED"]]),
            "baseline_power_cap_matched": bool(to[TO["BASE_CAP_MATCHED"]]),
            "baseline_state_matched": bool(to[TO["BASE_STATE_MATCHED"]]),
            "baseline_clock_domains_compared": ["graphics_clock_mhz", "memory_clock_mhz"] + (["sm_clock_mhz"] if to[TO["BASE_SM_COMPARED"]] else []),
            "baseline_sm_clock_uses_graphics_proxy": not bool(to[TO["BASE_SM_COMPARED"]]),
            "baseline_state_domains_compared": sorted(([ "enforced_power_limit_w"] if to[TO["BASE_ENF_COMPARED"]] else [])
                                                      + (["pstate"] if to[TO["BASE_PSTATE_COMPARED"]] else [])),
            "policy": dict(policy_dict), "phases": {},
        }
        # insertion order of the reference: idle_pre before idle_post, enforced limit before pstate (= bit order)
        result["baseline_state_issues"] = [s for s in baseline_issues if s.startswith("idle_state_mismatch_or_unverified")]
        result["active_minus_idle_state_deltas"] = _state_deltas(to, TO)
        tensor, memory = workload in TENSOR_WORKLOADS, workload in MEMORY_WORKLOADS
        result["total_pj_per_flop"] = g("TOTAL_PJ_PER_FLOP")
        result["total_pj_per_logical_bit"] = g("TOTAL_PJ_PER_BIT")
        result["operational_idle_increment_pj_per_flop"] = g("INC_PJ_PER_FLOP")
        result["operational_idle_increment_pj_per_logical_bit"] = g("INC_PJ_PER_BIT")
        result["flop_count_convention"] = "multiply-add=2 FLOPs; reported dense FP16 tensor operations" if tensor else None
        result["logical_bit_count_convention"] = "8 bits per logical byte; copy counts both read and write payload" if memory else None
        for name in ("idle_pre", "measure", "idle_post"):
            result["phases"][name] = phase_dicts[name]
        if phases_rec.get("active_control"):
            result["phases"]["active_control"] = phase_dicts["active_control"]
            result["active_control_incremental_power_w"] = g("CONTROL_INC_POWER_W")
            result["control_subtracted_power_w"] = None
        # paired reference
        result.update(paired_active_reference_eligible=bool(to[TO["PAIRED_ELIGIBLE"]]) and not paired_issues,
                      paired_active_reference_power_w=None, paired_active_reference_energy_j=None,
                      paired_active_reference_pj_per_flop=None, paired_active_reference_pj_per_logical_bit=None,
                      paired_active_reference_issues=sorted(set(paired_issues)),
                      paired_active_reference_protocol=record.get("treatment_protocol") or bench.get("treatment_protocol") or {})
        if phases_rec.get("active_reference"):
            result["paired_active_reference_eligible"] = (result["paired_active_reference_eligible"] and result["valid"])
            result.update(paired_active_reference_power_w=g("PAIRED_POWER_W"),
                          paired_active_reference_energy_j=g("PAIRED_ENERGY_J"),
                          paired_active_reference_pj_per_flop=g("PAIRED_PJ_PER_FLOP"),
                          paired_active_reference_pj_per_logical_bit=g("PAIRED_PJ_PER_BIT"),
                          paired_active_reference_drift_adjusted_power_w=g("PAIRED_DRIFT_ADJUSTED_W"),
                          active_reference_power_w=g("REF_POWER_W"), active_reference_duration_s=g("REF_DURATION_S"),
                          active_reference_total_energy_j=g("REF_TOTAL_ENERGY_J"),
                          paired_active_reference_state_deltas=_paired_deltas(to, TO))
            result["phases"]["active_reference"] = phase_dicts["active_reference"]
            result["paired_reference_clock_domains_compared"] = (["graphics_clock_mhz", "memory_clock_mhz"]
                                                                 + (["sm_clock_mhz"] if to[TO["PAIRED_SM_COMPARED"]] else []))
            result["paired_reference_sm_clock_uses_graphics_proxy"] = not bool(to[TO["PAIRED_SM_COMPARED"]])
        else:
            result["paired_active_reference_issues"] = ["missing_paired_active_reference_phase"]
            result["paired_active_reference_eligible"] = False
        if workload in SFU_WORKLOADS:
            rate = g("SFU_RATE")
            result.update(throughput_sfu_instructions_s=rate, counted_measure_sfu_instructions=g("SFU_COUNTED"),
                          pj_per_op=None, total_pj_per_op=None,
                          total_pj_per_instruction=g("SFU_TOTAL_PJ"),
                          operational_idle_increment_pj_per_instruction=g("SFU_INC_PJ"),
                          paired_active_reference_pj_per_instruction=g("SFU_PAIRED_PJ"),
                          sfu_reference_delta_pj_per_instruction=g("SFU_PAIRED_PJ"),
                          sfu_reference_delta_power_w=result.get("paired_active_reference_power_w"),
                          sfu_reference_delta_measurement_valid=result["paired_active_reference_eligible"],
                          sfu_reference_delta_issues=sorted(set(result["paired_active_reference_issues"]
                                                                + ["treatment:" + s for s in result["issues"]])))
            if phases_rec.get("active_reference"):
                result["active_reference_counted_loop_slots"] = g("REF_SLOTS")
                result["active_reference_loop_slots_s"] = g("REF_SLOTS_RATE")
        nonlinear = workload in NONLINEAR_WORKLOADS
        result.update(throughput_elements_s=g("ELEMENT_RATE"), throughput_rows_s=g("ROW_RATE"),
                      row_width=bench.get("row_width") if nonlinear else None,
                      counted_measure_elements=g("COUNTED_ELEMENTS"),
                      total_pj_per_element=g("PJ_ELEMENT_TOTAL"), operational_idle_increment_pj_per_element=g("PJ_ELEMENT_INC"),
                      paired_active_reference_pj_per_element=g("PJ_ELEMENT_PAIRED"),
                      total_pj_per_row=g("PJ_ROW_TOTAL"), operational_idle_increment_pj_per_row=g("PJ_ROW_INC"),
                      paired_active_reference_pj_per_row=g("PJ_ROW_PAIRED"))
        if nonlinear and g("ELEMENT_RATE") is None:
            result["pj_per_op"] = result["total_pj_per_op"] = None
        selected = _selected(packed, i, 1, views)
        result["hbm_bandwidth"] = trial_bandwidth(record, result, selected, hbm_bandwidth_fraction)
        sensor = trial_sensor(record, result, result["phases"], phases_rec, policy.max_sample_gap_s,
                              policy.max_idle_drift_fraction)
        result["hbm_memory_power"] = sensor
        if sensor is not None:
            for alias, field in SENSOR_ALIASES:
                result[alias] = sensor[field]
            if _metrics_out is not None:
                rows = _metrics_out[-1][0]
                for alias in ("memory_rail_power_w", "memory_rail_incremental_power_w"):
                    value = result[alias]
                    rows[i, METRICS.index(alias)] = math.nan if value is None else value
        reported = [p for p, name in enumerate(N.PHASE_NAMES)
                    if name in ("idle_pre", "measure", "idle_post") or (name == "active_control" and phases_rec.get(name))]
        complete_trial(record, result, policy.trim_s, _binding(packed, i, views),
                       _rail_sources(packed, i, reported, views))
        out.append(result)
    return out


def _windows(views) -> list:
    """Every slot's selected window (lo, hi) relative to its segment, or None: read from the
    phase rows at once."""
    rows = views.phase_out.reshape(-1, views.PO)
    pairs = rows[:, [N.layout("PM_PO_SEL_LO"), N.layout("PM_PO_SEL_HI")]].tolist()
    return [None if math.isnan(lo) else (int(lo), int(hi)) for lo, hi in pairs]


def _window(trial, phase, views):
    slot = trial * N.PM_PHASES + phase
    if views.windows is None:
        views.windows = _windows(views)
    return slot, views.windows[slot]


def _binding(packed, trial, views):
    """The measure window's clock bindings, built by the native packer."""
    from .pack import _native_packer
    slot, window = _window(trial, 1, views)
    if not window:
        return []
    if packed.clock_repeat is None:
        return _native_packer().binding_samples(packed.samples[slot], *window)
    offsets = packed.arrays["phase_offsets"]
    repeat = memoryview(packed.clock_repeat)[int(offsets[slot]):int(offsets[slot + 1])]
    return _native_packer().binding_samples(packed.samples[slot], *window, repeat)


def _rail_sources(packed, trial, phases, views):
    """Memory-power sources of the selected windows; the packed flag words say first whether any
    selected sample reports a memory power at all."""
    from .trial_report import rail_sources_of
    flags, offsets = packed.arrays["sample_flags"], packed.arrays["phase_offsets"]
    windows = []
    for p in phases:
        slot, window = _window(trial, p, views)
        if window:
            windows.append((slot, window))
    if packed.broadcast & dict(N.BROADCAST_COLUMNS)["sample_flags"]:        # one flag word for every sample
        any_memory = bool(windows) and bool(int(flags[0]) & N.S_MEMORY_POWER_SET)
    else:
        any_memory = any((flags[offsets[slot] + a:offsets[slot] + b] & N.S_MEMORY_POWER_SET).any() for slot, (a, b) in windows)
    if not any_memory:
        return []
    return rail_sources_of(packed.samples[slot][a:b] for slot, (a, b) in windows)


def _selected(packed, trial, phase, views):
    slot, window = _window(trial, phase, views)
    return packed.samples[slot][window[0]:window[1]] if window else []


_TO_NAMES = ("DURATION_S", "BENCH_MEASURED_DURATION_S", "BENCH_DEVICE_DURATION_S", "IDLE_POWER_W", "IDLE_MEMORY_POWER_W",
             "TOTAL_ENERGY_J", "ENERGY_SOURCE_TRAPEZOID", "BOARD_POWER_W", "IDLE_ENERGY_J", "INCREMENTAL_ENERGY_J",
             "INCREMENTAL_POWER_W", "OPS_RATE", "BYTE_RATE", "DEVICE_OPS_RATE", "DEVICE_BYTE_RATE", "COUNTED_OPS",
             "COUNTED_BYTES", "EPOCHS", "EXACT", "RAIL_ENERGY_J", "RAIL_INCREMENTAL_J", "RAIL_INCREMENTAL_W",
             "POWER_LIMIT_W", "TENSOR_PEAK_TFLOPS", "PEAK_CLOCK_IS_SM", "TENSOR_UTILIZATION", "IDLE_FRAC_MEASURED",
             "IDLE_FRAC_LIMIT", "LIMIT_UTILIZATION", "PJ_PER_OP", "PJ_PER_LOGICAL_BYTE", "TOTAL_PJ_PER_OP",
             "TOTAL_PJ_PER_LOGICAL_BYTE", "TOTAL_PJ_PER_FLOP", "TOTAL_PJ_PER_BIT", "INC_PJ_PER_FLOP", "INC_PJ_PER_BIT",
             "BASE_CLOCK_MATCHED", "BASE_TEMP_MATCHED", "BASE_CAP_MATCHED", "BASE_STATE_MATCHED", "BASE_SM_COMPARED",
             "BASE_ENF_COMPARED", "BASE_PSTATE_COMPARED", "DPRE_GFX", "DPRE_MEM", "DPRE_SM", "DPRE_TEMP", "DPRE_ENF",
             "DPRE_PSTATE", "DPOST_GFX", "DPOST_MEM", "DPOST_SM", "DPOST_TEMP", "DPOST_ENF", "DPOST_PSTATE",
             "PAIRED_POWER_W", "PAIRED_ENERGY_J", "PAIRED_ELIGIBLE", "REF_POWER_W", "REF_DURATION_S", "REF_TOTAL_ENERGY_J",
             "PAIRED_PJ_PER_FLOP", "PAIRED_PJ_PER_BIT", "PAIRED_DRIFT_ADJUSTED_W", "PAIRED_D_GFX", "PAIRED_D_MEM",
             "PAIRED_D_SM", "PAIRED_D_TEMP", "PAIRED_SM_COMPARED", "REF_SLOTS", "REF_SLOTS_RATE", "SFU_RATE",
             "SFU_COUNTED", "SFU_TOTAL_PJ", "SFU_INC_PJ", "SFU_PAIRED_PJ", "ELEMENT_RATE", "ROW_RATE", "COUNTED_ELEMENTS",
             "PJ_ELEMENT_TOTAL", "PJ_ELEMENT_INC", "PJ_ELEMENT_PAIRED", "PJ_ROW_TOTAL", "PJ_ROW_INC", "PJ_ROW_PAIRED",
             "CONTROL_INC_POWER_W", "VALID", "BASELINE_VALID", "IDLE_INC_ELIGIBLE", "THROTTLE_MASK")


def _state_deltas(to, TO):
    out = {}
    sm = bool(to[TO["BASE_SM_COMPARED"]])
    for name, prefix in (("idle_pre", "DPRE"), ("idle_post", "DPOST")):
        d = {"graphics_clock_mhz": _none(to[TO[prefix + "_GFX"]]), "memory_clock_mhz": _none(to[TO[prefix + "_MEM"]])}
        if sm:
            d["sm_clock_mhz"] = _none(to[TO[prefix + "_SM"]])
        d["temperature_c"] = _none(to[TO[prefix + "_TEMP"]])
        if to[TO["BASE_ENF_COMPARED"]]:
            d["enforced_power_limit_w"] = _none(to[TO[prefix + "_ENF"]])
        if to[TO["BASE_PSTATE_COMPARED"]]:
            d["pstate"] = _none(to[TO[prefix + "_PSTATE"]])
        out[name] = d
    return out


def _paired_deltas(to, TO):
    d = {"graphics_clock_mhz": _none(to[TO["PAIRED_D_GFX"]]), "memory_clock_mhz": _none(to[TO["PAIRED_D_MEM"]])}
    if to[TO["PAIRED_SM_COMPARED"]]:
        d["sm_clock_mhz"] = _none(to[TO["PAIRED_D_SM"]])
    d["temperature_c"] = _none(to[TO["PAIRED_D_TEMP"]])
    return d


def analyze_trial(record: Mapping[str, Any], policy: AnalysisPolicy | Mapping[str, Any] | None = None,
                  hbm_bandwidth_fraction: float = 0.80) -> dict[str, Any]:
    """One trial through the batched kernel (analysis.py:597 interface)."""
    return analyze_trials([record], policy, hbm_bandwidth_fraction)[0]


def group_key(trial: Mapping[str, Any]) -> str:
    """The reference's _group_key (analysis.py:1078-1093): its sha256 seeds the group's resampling."""
    config = {k: v for k, v in trial.get("config", {}).items() if k not in REPEAT_KEYS}
    achieved = None if trial.get("clock_comparison_controlled") else {
        f: trial.get(f) for f in ("graphics_clock_mhz", "memory_clock_mhz")}
    from .trial_report import _record_native
    # json.dumps(..., sort_keys=True, separators=(",", ":")), written natively
    return _record_native().sorted_json({"gpu_uuid": trial.get("gpu_uuid"), "workload": trial.get("workload"),
                       "experiment_role": trial.get("experiment_role", "legacy_unspecified"),
                       "config": config, "uncontrolled_achieved_clocks": achieved,
                       "benchmark_sha256": trial.get("benchmark_sha256"),
                       "measurement_stratum": trial.get("measurement_stratum"),
                       "experiment_contract": trial.get("experiment_contract"),
                       "nonlinear_contract": trial.get("nonlinear_contract"),
                       "sfu_contract": trial.get("sfu_contract"),
                       "treatment_design_stratum": trial.get("treatment_design_stratum"),
                       "resource_geometry": trial.get("resource_geometry")})


def group_seed(key: str) -> int:
    return int(hashlib.sha256(key.encode()).hexdigest()[:16], 16)


def bootstrap_groups(values: np.ndarray, members: list[list[int]], seeds: list[int],
                     resamples: int = DEFAULT_RESAMPLES) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Medians and CIs of ``values[rows, metrics]`` for each group's member rows, on the GPU."""
    values = np.ascontiguousarray(values, dtype=np.float64)
    n_rows, n_metrics = values.shape
    offsets = np.zeros(len(members) + 1, dtype=np.int32)
    np.cumsum([len(m) for m in members], out=offsets[1:])
    rows = np.ascontiguousarray(np.concatenate([np.asarray(m, dtype=np.int32) for m in members]) if members else np.zeros(0, np.int32))
    seeds_a = np.asarray(seeds, dtype=np.uint64)
    G = len(members)
    med, lo, hi = (np.empty((G, n_metrics)) for _ in range(3))
    job = N.BootstrapJob(G, n_metrics, int(rows.size), n_rows, resamples, max((len(m) for m in members), default=0),
                         values.ctypes.data, offsets.ctypes.data, rows.ctypes.data if rows.size else None, None,
                         seeds_a.ctypes.data if G else None, med.ctypes.data, lo.ctypes.data, hi.ctypes.data)
    N.check(N.library().pm_group_bootstrap(job), "pm_group_bootstrap")
    return med, lo, hi


def median_ci(values: list[float], seed: int, resamples: int = DEFAULT_RESAMPLES) -> list[float] | None:
    """_median_ci (analysis.py:1096-1101) for one value list, on the GPU."""
    if len(values) < 3:
        return None
    _, lo, hi = bootstrap_groups(np.asarray(values, dtype=np.float64).reshape(-1, 1), [list(range(len(values)))], [seed], resamples)
    return [float(lo[0, 0]), float(hi[0, 0])]


def dedup_trials(records: list) -> tuple[list, list]:
    """Records kept (first of each trial_id) and the duplicate ids dropped (analysis.py:1408-1416)."""
    seen, duplicates, kept = set(), [], []
    for record in records:
        trial_id = record.get("trial_id")
        if trial_id is not None and trial_id in seen:
            duplicates.append(trial_id)
            continue
        if trial_id is not None:
            seen.add(trial_id)
        kept.append(record)
    return kept, duplicates


def analyze_rows(records: list, policy: AnalysisPolicy, hbm_bandwidth_fraction: float) -> tuple[list, np.ndarray]:
    """Trial results plus one row per trial: the 47 metrics, then the 7 memory-rail sensor fields.

    The sensor columns are NaN outside each field's repeat population, so the
    bootstrap of an HBM group's sensor fields (memory_power.py:169-204) runs
    in the same launch as its metrics.
    """
    metrics_out: list = []
    trials = analyze_trials(records, policy, hbm_bandwidth_fraction, _metrics_out=metrics_out)
    metric_rows = metrics_out[0][0] if metrics_out else np.zeros((0, len(METRICS)))
    sensor_rows = np.array([sensor_columns(t.get("hbm_memory_power")) for t in trials], dtype=np.float64)
    rows = np.concatenate([metric_rows, sensor_rows.reshape(len(trials), len(SENSOR_FIELDS))], axis=1)
    return trials, rows


def group_structure(trials: list, min_repeats: int) -> tuple[list, list, list, list]:
    """Groups in key order with their valid members, seeds and all members (analysis.py:1424-1466)."""
    buckets: dict[str, list[int]] = {}
    for index, trial in enumerate(trials):
        buckets.setdefault(group_key(trial), []).append(index)
    ordered = sorted(buckets.items())
    members, seeds, groups, group_indices = [], [], [], []
    for key, indices in ordered:
        group_indices.append(indices)
        valid, seen_repeats, dup_repeats = [], set(), []
        for index in indices:
            trial = trials[index]
            if not trial["valid"]:
                continue
            repeat = trial.get("repeat_index")
            if repeat is not None and repeat in seen_repeats:
                dup_repeats.append(repeat)
                continue
            if repeat is not None:
                seen_repeats.add(repeat)
            valid.append(index)
        digest = hashlib.sha256(key.encode()).hexdigest()[:16]
        members.append(valid)
        seeds.append(int(digest, 16))
        first = trials[indices[0]]
        vt = [trials[i] for i in valid]
        group = {"group_id": digest, "gpu_uuid": first["gpu_uuid"], "workload": first["workload"],
                 "experiment_role": first.get("experiment_role", "legacy_unspecified"),
                 "experiment_contract": first.get("experiment_contract"),
                 "nonlinear_contract": first.get("nonlinear_contract"), "sfu_contract": first.get("sfu_contract"),
                 "config": {k: v for k, v in first["config"].items() if k not in REPEAT_KEYS},
                 "benchmark_sha256": first["benchmark_sha256"], "measurement_stratum": first["measurement_stratum"],
                 "kernel_implementation_version": first.get("kernel_implementation_version"),
                 "treatment_design_stratum": first["treatment_design_stratum"],
                 "resource_geometry": first["resource_geometry"],
                 "repeats": len(indices), "valid_repeats": len(valid), "trial_ids": [trials[i]["trial_id"] for i in indices],
                 "duplicate_repeat_indices_ignored": dup_repeats,
                 "target_verified": False, "verified_selection_eligible": False,
                 "count_energy_time_alignment_exact": bool(vt) and all(t["count_energy_time_alignment_exact"] for t in vt),
                 "clock_comparison_controlled": bool(vt) and all(t["clock_comparison_controlled"] for t in vt),
                 "diagnostic_only": first["diagnostic_only"], "gpu_name": first["gpu_name"],
                 "baseline_valid": bool(vt) and all(t["baseline_valid"] for t in vt),
                 "operational_idle_increment_eligible": bool(vt) and all(t["operational_idle_increment_eligible"] for t in vt),
                 "paired_active_reference_eligible": bool(vt) and all(t["paired_active_reference_eligible"] for t in vt),
                 "paired_reference_order_counts": {o: sum((t.get("paired_active_reference_protocol") or {}).get("order") == o for t in vt)
                                                   for o in ("AB", "BA")},
                 "confidence": "repeat_median" if len(valid) >= min_repeats else "insufficient_valid_repeats", "ci95": {}}
        groups.append(group)
    return groups, members, seeds, group_indices


def finish_groups(groups: list, trials: list, members: list, group_indices: list, med: np.ndarray, lo: np.ndarray,
                  hi: np.ndarray, hbm_bandwidth_fraction: float, min_repeats: int = 3) -> None:
    """Group medians, intervals and the derived group records, from the bootstrap outputs (in place)."""
    from .hbm import group_bandwidth
    from .trial_report import complete_group
    base = len(METRICS)
    if not groups:
        return
    # the bootstrap outputs as rows of Python floats, None for NaN, converted at once
    width = med.shape[1]
    med_rows, lo_rows, hi_rows = (_py_rows(np.ascontiguousarray(x).reshape(-1), width) for x in (med, lo, hi))
    for g, group in enumerate(groups):
        mr, lr, hr = med_rows[g], lo_rows[g], hi_rows[g]
        ci = group["ci95"]
        for m, metric in enumerate(METRICS):
            group[metric] = mr[m]
            a = lr[m]
            ci[metric] = [a, hr[m]] if a is not None else None
        vt = [trials[i] for i in members[g]]
        group["hbm_bandwidth"] = group_bandwidth(vt, group["workload"], hbm_bandwidth_fraction)
        sensor_medians = mr[base:base + len(SENSOR_FIELDS)]
        sensor_intervals = [[lr[base + k], hr[base + k]] if lr[base + k] is not None else None
                            for k in range(len(SENSOR_FIELDS))]
        group["hbm_memory_power"] = group_sensor(vt, group["workload"], [trials[i] for i in group_indices[g]],
                                                 sensor_medians, sensor_intervals)
        if group["hbm_memory_power"] is not None:
            sensor = group["hbm_memory_power"]
            for alias, field in SENSOR_ALIASES:
                group[alias] = sensor[field]
                group["ci95"][alias] = sensor["ci95"][field]
        counts = group["paired_reference_order_counts"]
        group["paired_reference_both_orders_observed"] = all(counts.values())
        group["paired_reference_counterbalanced"] = group["paired_reference_both_orders_observed"] and counts["AB"] == counts["BA"]
        group["paired_reference_order_count_imbalance"] = counts["AB"] - counts["BA"]
        group["paired_active_reference_eligible"] = group["paired_active_reference_eligible"] and group["paired_reference_counterbalanced"]
        arm = {}
        for order in ("AB", "BA"):
            vals = [v for t in vt if (t.get("paired_active_reference_protocol") or {}).get("order") == order
                    and (v := finite(t.get("paired_active_reference_power_w"))) is not None]
            arm[order] = statistics.median(vals) if vals else None
        group["paired_reference_order_medians_power_w"] = arm
        group["paired_reference_order_effect_power_w"] = arm["AB"] - arm["BA"] if None not in arm.values() else None
        complete_group(group, trials[group_indices[g][0]], vt, min_repeats)


NOTES = ["No fabricated measurement or architecture-specific idle wattage is supplied.",
         "A device power limit is not measured consumption, and headline FLOP/s is not achieved throughput.",
         "Idle subtraction cannot separate physical static leakage from refresh/clock/background power.",
         "L1/L2/HBM logical bytes are not guaranteed physical traffic; numeric profiler evidence is recomputed for target verification.",
         "Verified selections require exact matching work/power windows; old records retain explicitly qualified stationary-rate estimates.",
         "Uncontrolled default-clock trials are comparative and excluded from controlled-frequency optimum searches.",
         "Each GPU UUID has its own empirically selected optimum; 1110 MHz is a mandatory supported sweep point, not a preset optimum.",
         "Near-optimum and uncertainty-overlap sets contain only measured support points; no continuous interval or unmeasured gap is claimed."]
"""The summary's notes (analysis.py:1547-1554), reported as the reference reports them."""


def summary_record(trials: list, groups: list, duplicates: list, throughput_fraction: float,
                   hbm_bandwidth_fraction: float, min_repeats: int, resamples: int,
                   policy: AnalysisPolicy | None = None) -> dict[str, Any]:
    """The summary: trials, groups, and the selection sections over the groups (analysis.py:1500-1556)."""
    from . import selections as S
    policy = policy or AnalysisPolicy()
    f, n = throughput_fraction, min_repeats
    optima = lambda across, single: S.energy_optima(  # noqa: E731
        groups, f, n, policy.near_optimum_fraction, policy.min_geometries, across_memory_domains=across,
        single_geometry_exploratory=single)
    with S.stratum_memo():
        return _summary_sections(S, trials, groups, duplicates, f, n, optima, hbm_bandwidth_fraction, policy, resamples)


def _summary_sections(S, trials, groups, duplicates, f, n, optima, hbm_bandwidth_fraction, policy, resamples):
    return {"schema_version": 2, "trials": trials, "groups": groups, "duplicate_trial_ids_ignored": duplicates,
            "within_clock_best": S.best_conditions(groups, f, n, False),
            "cross_clock_best": S.best_conditions(groups, f, n, True),
            "within_clock_best_total_energy": S.best_conditions(groups, f, n, False, total_energy=True),
            "cross_clock_best_total_energy": S.best_conditions(groups, f, n, True, total_energy=True),
            "uncontrolled_clock_exploratory_best": S.best_conditions(groups, f, n, True, exploratory_only=True),
            "pareto_frontiers": S.pareto_frontiers(groups, n, False) + S.pareto_frontiers(groups, n, True),
            "active_control_associations": S.control_associations(groups, n),
            "verified_target_within_clock_best": S.best_conditions(groups, f, n, False, True),
            "verified_target_cross_clock_best": S.best_conditions(groups, f, n, True, True),
            "verified_target_coverage": S.verification_coverage(groups, f, n, False) + S.verification_coverage(groups, f, n, True),
            "empirical_gpu_energy_optima": optima(False, False),
            "empirical_gpu_overall_energy_optima": optima(True, False),
            "exploratory_single_geometry_energy_optima": optima(False, True),
            "exploratory_single_geometry_overall_energy_optima": optima(True, True),
            "metric_aliases": {"pj_per_op": "legacy operational idle increment per reported benchmark operation; tensor FLOP uses explicit operational_idle_increment_pj_per_flop",
                               "pj_per_logical_byte": "legacy operational idle increment per logical byte; divide by 8 for logical-bit metric",
                               "incremental_power_w": "operational_idle_increment_power_w; a baseline contrast, not physical switching power"},
            "selection_policy": {"throughput_fraction": f, "hbm_bandwidth_fraction": hbm_bandwidth_fraction,
                                 "hbm_throughput_constraint": "all conditions with median sustained logical bandwidth >= the configured fraction of clock-specific DDR theory; every valid repeat needs complete measured memory-clock and CUDA bus-width evidence; observed 95% and plateaus are diagnostic only",
                                 "min_repeats": n, "min_geometries": policy.min_geometries,
                                 "near_optimum_fraction": policy.near_optimum_fraction,
                                 "geometry_requirement": "at least min_geometries distinct verified execution-resource geometries per frequency; throughput peak still uses all valid groups; repeat/seed/footprint-only variants do not qualify; count alone is not saturation proof",
                                 "primary_energy_objective": "whole-device total energy per logical bit, FLOP or nonlinear output element",
                                 "frequency_utilization_constraint": "HBM: clock-specific theoretical bandwidth gate; other workloads: own-frequency complete measured geometry peak, with global-near-peak optima reported separately",
                                 "baseline_objectives": "separate matched operational idle increment and paired active-reference contrast; never automatically substituted for total energy",
                                 "ci_method": f"deterministic percentile bootstrap of repeat medians ({resamples} draws); n=3 intervals are coarse"},
            "notes": list(NOTES)}


def check_summary_arguments(throughput_fraction: float, min_repeats: int, hbm_bandwidth_fraction: float) -> float:
    if not 0 < throughput_fraction <= 1 or min_repeats < 1:
        raise ValueError("throughput_fraction must be in (0, 1], min_repeats must be positive")
    from .hbm import validate_fraction
    return validate_fraction(hbm_bandwidth_fraction)


def summarize(records: Iterable[Mapping[str, Any]], throughput_fraction: float = 0.95,
              policy: AnalysisPolicy | Mapping[str, Any] | None = None, min_repeats: int = 3,
              plan: Mapping[str, Any] | None = None, evaluation_policy=None,
              hbm_bandwidth_fraction: float = 0.80, resamples: int = DEFAULT_RESAMPLES,
              plan_validator=None) -> dict[str, Any]:
    """The reference's summary (analysis.py:1400-1556): trials, groups, selection sections and the
    component evaluation; ``resamples`` generalises the 1000 draws.  ``plan`` and
    ``evaluation_policy`` go to the evaluation (powermodeling_b200.evaluation.evaluate), whose
    planner policy check is not restated: pass ``plan_validator`` (runner.validate_plan_execution)
    to have its error recorded in the coverage.

    The cyclic garbage collector is paused for the call: the summary is built
    from tens of thousands of new dicts and lists, and a full collection in
    the middle would walk every sample dict of the records (over 200 000 for
    a 64-point sweep) for nothing, tripling the call's time."""
    paused = gc.isenabled()
    gc.disable()
    try:
        records = records if isinstance(records, list) else list(records)
        summary = _summarize(records, throughput_fraction, policy, min_repeats, hbm_bandwidth_fraction, resamples)
        from .evaluation import evaluate
        summary["evaluation"] = evaluate(summary, plan=plan, policy=evaluation_policy, raw_records=records,
                                         plan_validator=plan_validator)
        return summary
    finally:
        if paused:
            gc.enable()


def _summarize(records, throughput_fraction, policy, min_repeats, hbm_bandwidth_fraction, resamples) -> dict[str, Any]:
    hbm_bandwidth_fraction = check_summary_arguments(throughput_fraction, min_repeats, hbm_bandwidth_fraction)
    policy = _policy(policy)
    kept, duplicates = dedup_trials(list(records))
    trials, rows = analyze_rows(kept, policy, hbm_bandwidth_fraction)
    groups, members, seeds, group_indices = group_structure(trials, min_repeats)
    med, lo, hi = bootstrap_groups(rows, members, seeds, resamples) if groups else (None, None, None)
    finish_groups(groups, trials, members, group_indices, med, lo, hi, hbm_bandwidth_fraction, min_repeats)
    return summary_record(trials, groups, duplicates, throughput_fraction, hbm_bandwidth_fraction, min_repeats,
                          resamples, policy)


# trials.csv columns (analysis.py:1565-1573), in the reference's order.
TRIAL_CSV_FIELDS = (
    "trial_id", "gpu_uuid", "gpu_name", "workload", "experiment_role", "valid", "target_verified", "ncu_status",
    "ncu_target_suitability", "ncu_utilization_status", "profiler_suitability_status", "memory_access_geometry",
    "memory_coalescing", "memory_coalescing_energy_eligible", "energy_peak_population_eligible",
    "verified_selection_eligible", "count_energy_time_alignment_exact", "energy_per_work_kind", "issues", "warnings",
    "baseline_valid", "baseline_issues", "operational_idle_increment_eligible", "paired_active_reference_eligible",
    "paired_active_reference_issues", "treatment_design_stratum", "baseline_clock_domains_compared",
    "baseline_sm_clock_uses_graphics_proxy", "baseline_state_matched", "baseline_state_issues",
    "baseline_state_domains_compared", "resource_geometry", "row_width", "nonlinear_contract",
    "counted_measure_elements", "element_count_convention", "row_operation_convention",
    "paired_reference_clock_domains_compared", "paired_reference_sm_clock_uses_graphics_proxy", "duration_s", *METRICS,
    "total_energy_j", "incremental_energy_j", "energy_source", "power_limit_w", "tensor_peak_clock_source",
    "hbm_memory_power", "hbm_bandwidth", "memory_rail_energy_j", "memory_rail_idle_power_w",
    "memory_rail_incremental_energy_j", "memory_rail_sources",
    "sfu_contract", "counted_measure_sfu_instructions", "sfu_instruction_count_convention",
    "sfu_reference_delta_measurement_valid", "sfu_reference_delta_positive_optimum_eligible",
    "sfu_reference_delta_estimator", "sfu_reference_delta_diagnostics", "sfu_reference_delta_issues",
    "sfu_hardware_attribution_proven")


def write_summary(summary: Mapping[str, Any], output_dir) -> dict[str, str]:
    """summary.json and trials.csv of a summary (analysis.py:1559-1583).

    summary.json is the summary as indented JSON (non-finite numbers refused,
    as the reference refuses them); trials.csv holds one row per trial with
    the reference's columns, lists and dicts as JSON text and absent fields
    empty.  A summary with an ``evaluation`` entry also gets evaluation.json,
    evaluation.csv and, with an HBM component, hbm-memory-power.csv
    (evaluation.write_evaluation; the reference's HTML view is not written)."""
    import csv
    from pathlib import Path
    destination = Path(output_dir)
    destination.mkdir(parents=True, exist_ok=True)
    json_path = destination / "summary.json"
    json_path.write_text(json.dumps(summary, indent=2, ensure_ascii=False, allow_nan=False) + "\n")
    csv_path = destination / "trials.csv"
    with csv_path.open("w", newline="") as stream:
        writer = csv.DictWriter(stream, fieldnames=TRIAL_CSV_FIELDS)
        writer.writeheader()
        for trial in summary.get("trials", []):
            writer.writerow({f: json.dumps(trial[f]) if isinstance(trial.get(f), (list, dict)) else trial.get(f)
                             for f in TRIAL_CSV_FIELDS})
    paths = {"summary_json": str(json_path), "trials_csv": str(csv_path)}
    if summary.get("evaluation") is not None:
        from .evaluation import write_evaluation
        paths.update(write_evaluation(summary["evaluation"], destination))
    return paths

