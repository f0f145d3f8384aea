"""The reporting half of a trial record: every field of the reference's
analyze_trial that follows from the record and the trial's numeric results
without further telemetry arithmetic (analysis.py:838-986 and 1000-1056, with
_physical_traffic_estimates 280-290, _paired_reference_contrast's SFU
diagnostics 392-415 and _measurement_diagnostics 433-565).

``complete_trial(record, result, ...)`` adds them to a result dict that
already holds the GPU's numbers (energies, powers, rates, eligibility, issues).
The fields fall in four kinds, each built by one function:

* ``_passthrough``: values copied from the record (kernel resources, feature
  and power provenance, the operation unit, latency probes ...);
* ``_statements``: fixed interpretive statements, some chosen by the trial's
  timebase or workload;
* ``_profiler_state``: the profiler admission when no numeric profiler
  evidence is attached (unprofiled, inconclusive) and the memory-read
  coalescing record that follows from the declared read geometry alone;
* ``measurement_diagnostics``: numerator, denominator and scope factors of
  each energy objective, recomputed from the reported fields.

Records that carry numeric profiler evidence (``validation.profiler_evidence``)
need the Nsight evidence assessor, which this package does not provide; they
are refused.
"""
from __future__ import annotations

import math
from typing import Any, Mapping

from .pack import MEMORY_WORKLOADS, NONLINEAR_WORKLOADS, ROW_WORKLOADS, SFU_WORKLOADS, TENSOR_WORKLOADS, finite
from .selections import ENERGY, peak_population_eligible, read_geometry, role_eligible

MISSING_EVIDENCE = {"status": "inconclusive", "suitable_verified": False,
                    "reasons": ["missing_numeric_profiler_evidence"], "checks": [], "kernels": []}

_TEXT = {
    "treatment_outcome_kind": "measured whole-device total energy per counted treatment work",
    "idle_baseline_estimator": "linear interpolation between pre/post trimmed idle mean power at treatment midpoint; integral exact for the assumed linear drift",
    "idle_increment_interpretation": "operational whole-device contrast against powered idle; activation, clock distribution, refresh and background changes may remain; physical leakage/switching are not isolated",
    "baseline_kind": "powered-idle baseline; includes leakage, clocks, refresh, and device background activity",
    "baseline_power_scope": "same measured device/API rail; idle is an operational state, not a leakage meter",
    "dynamic_attribution_note": "Eligibility indicates matched-baseline/profiler prerequisites only. It does not prove isolation of physical switching power or static leakage.",
    "attribution": "whole-device incremental energy per benchmark operation or logical byte; not isolated block energy",
}
_PAIRED_TEXT = ("same-process active issue-loop reference contrast; instruction, memory and scheduling differences "
                "remain; physical component switching power is not isolated")
_PAIRED_TEXT_SFU = ("signed whole-device power contrast against the target-free register recurrence; differing "
                    "instruction paths, issue rates, occupancy, launch work and epilogues remain; not isolated "
                    "physical SFU energy")
_CONTROL_NOTE = ("Standalone activation control is descriptive; paired protocol and state checks are required for an "
                 "active-reference contrast.")
_ELEMENT_CONVENTION = ("one output element of the complete FP32 function, including reductions/gamma and input/output; "
                       "not FLOPs or SFU instructions")
_ROW_CONVENTION = "one complete row function application; pJ/row = row_width * pJ/element"


def _passthrough(record: Mapping, bench: Mapping, device: Mapping) -> dict[str, Any]:
    workload = record.get("workload")
    carried = workload in NONLINEAR_WORKLOADS or workload in SFU_WORKLOADS
    out = {k: bench.get(k) for k in ("latency_probe", "kernel_resources", "execution_diagnostics",
                                     "memory_accesses_per_thread_iteration", "operation_unit")}
    out["numerical_validation"] = bench.get("numerical_validation") if carried else None
    out.update({k: record.get(k) for k in ("model_features", "feature_units", "feature_provenance", "power_provenance")})
    out["power_scope"] = (record.get("telemetry") or {}).get(
        "power_scope", device.get("power_scope_note", "NVML reported device power; scope depends on SKU/API"))
    out["power_usage_semantics"] = device.get("power_usage_semantics")
    return out


def _timebase(bench: Mapping, epochs: list) -> str:
    if epochs:
        return "complete monotonic work epochs with energy integrated over matching boundaries"
    if bench.get("host_duration_s"):
        return "estimated stationary rate from whole benchmark host duration"
    return "estimated stationary rate from whole benchmark duration; host timebase unavailable"


def _statements(record: Mapping, bench: Mapping, result: Mapping, epochs: list) -> dict[str, Any]:
    workload = record.get("workload")
    out = dict(_TEXT)
    out["throughput_timebase"] = _timebase(bench, epochs)
    out["paired_active_reference_interpretation"] = (
        _PAIRED_TEXT_SFU if workload in SFU_WORKLOADS and (result.get("phases") or {}).get("active_reference")
        else _PAIRED_TEXT)
    nonlinear = workload in NONLINEAR_WORKLOADS
    width = bench.get("row_width") if workload in ROW_WORKLOADS else None
    out["element_count_convention"] = _ELEMENT_CONVENTION if nonlinear else None
    out["row_operation_convention"] = _ROW_CONVENTION if width else None
    return out


def _coalescing(geometry: Mapping) -> dict[str, Any] | None:
    """The read-coalescing record of a trial without profiler evidence: it follows from the
    declared geometry, and no counter binds it (never energy-eligible)."""
    if geometry.get("applicable") is not True:
        return None
    record = {"applicable": True, "status": "inconclusive", "energy_eligible": False,
              "reasons": sorted(set(geometry.get("reasons", [])) | {"missing_bound_sector_counter_evidence"}),
              "geometry": geometry, "profile_binding_verified": False,
              "expected_sector_bytes_per_logical_read_byte": 1.0, "expected_sector_efficiency_fraction": 1.0,
              "requested_sector_efficiency_fraction": geometry.get("requested_sector_efficiency_fraction"),
              "observed_sector_bytes_per_logical_read_byte": None, "observed_sector_efficiency_fraction": None,
              "observed_sector_efficiency_pct": None, "counter_name": None, "counter_scope": None,
              "energy_denominator_use": "forbidden_separate_profiler_run", "profile_geometry": geometry}
    if geometry.get("status") == "fail":
        record["status"] = "fail"
    return record


def _profiler_state(record: Mapping, bench: Mapping, config: Mapping, result: Mapping) -> dict[str, Any]:
    provided = record.get("validation") or {}
    if isinstance(provided, dict) and isinstance(provided.get("profiler_evidence"), dict):
        raise ValueError("trial %r carries numeric profiler evidence; assessing it needs the Nsight evidence "
                         "assessor (validation.validate_evidence), which this package does not provide"
                         % (record.get("trial_id"),))
    workload = record.get("workload")
    geometry = read_geometry(bench, workload, config)
    coalescing = _coalescing(geometry)
    required = coalescing is not None
    coalescing_ok = not required                        # never energy-eligible without bound counters
    role_ok = role_eligible({"workload": workload, "experiment_role": record.get("experiment_role", "legacy_unspecified"),
                             "config": config, "experiment_contract": result.get("experiment_contract")})
    validation = {"assessment": dict(MISSING_EVIDENCE), "status": MISSING_EVIDENCE["status"], "profiler_evidence": None}
    if isinstance(provided, dict) and provided.get("locality"):
        validation["requested_locality"] = provided["locality"]
    return {"memory_access_geometry": geometry if workload in MEMORY_WORKLOADS else None,
            "memory_coalescing": coalescing, "memory_coalescing_energy_eligible": coalescing_ok if required else None,
            "target_verified": False, "validation": validation, "profile_rates_summary": None,
            "profiler_suitability_status": MISSING_EVIDENCE["status"], "ncu_status": "unprofiled",
            "ncu_assessment": dict(MISSING_EVIDENCE), "ncu_target_suitability": False,
            "ncu_utilization_status": "inconclusive",
            "verified_selection_eligible": False,             # target evidence is required
            "dynamic_attribution_eligible": False,
            "diagnostic_only": workload not in ENERGY or not role_ok,
            "physical_traffic_energy": {
                "physical_pj_per_bit": None,
                "status": "unavailable_without_matched_energy_window_hardware_traffic_counts", "profile_rates": None,
                "note": "Nsight replay busy-time rates and logical/physical ratios are diagnostic; they are not the energy-window physical-bit denominator."}}


def kept_epochs(bench: Mapping, phase: Mapping | None, trim_s: float) -> list[dict]:
    """The complete work epochs inside the trimmed measure window, in time order (for a trial whose
    epochs the analysis accepted: the parse cannot fail here)."""
    source = bench.get("measure_epochs", bench.get("work_epochs")) or []
    start, end = finite((phase or {}).get("start_s")), finite((phase or {}).get("end_s"))
    parsed = []
    for epoch in source:
        a, b = finite(epoch.get("start_s")), finite(epoch.get("end_s"))
        if a is None:
            stamp = finite(epoch.get("host_monotonic_start_ns", epoch.get("start_ns")))
            a = stamp / 1e9 if stamp is not None else None
        if b is None:
            stamp = finite(epoch.get("host_monotonic_end_ns", epoch.get("end_ns")))
            b = stamp / 1e9 if stamp is not None else None
        parsed.append({**epoch, "start_s": a, "end_s": b})
    parsed.sort(key=lambda e: e["start_s"])
    return [e for e in parsed if e["start_s"] >= start + trim_s - 1e-6 and e["end_s"] <= end - trim_s + 1e-6]


def binding_samples(selected: list) -> list[dict]:
    """The measure window's clock bindings (the native packer builds the same list faster)."""
    return [{"phase": "measure", "graphics_clock_mhz": s.get("graphics_clock_mhz"),
             "memory_clock_mhz": s.get("memory_clock_mhz")} for s in selected]


def _validation_binding(record: Mapping, bench: Mapping, config: Mapping, binding: list) -> dict[str, Any]:
    return {"condition_id": record.get("condition_id"), "workload": record.get("workload"), "config": config,
            "provenance": record.get("provenance"),
            "benchmark": {k: v for k, v in bench.items() if k not in ("measure_epochs", "work_epochs")},
            "samples": binding}


def _sfu_diagnostics(record: Mapping, bench: Mapping, result: dict, count_ok: bool) -> None:
    """The SFU paired-contrast diagnostics (present with an active reference arm)."""
    reference = record.get("active_reference") or {}
    ref_phase = (result.get("phases") or {}).get("active_reference") or {}
    rate = result.get("throughput_sfu_instructions_s")
    counted = result.get("counted_measure_operations")
    slots = result.get("active_reference_counted_loop_slots")
    slots_rate = result.get("active_reference_loop_slots_s")
    reference_power = result.get("active_reference_power_w")
    contrast = result.get("paired_active_reference_power_w")
    result["sfu_reference_delta_diagnostics"] = {
        "estimator": "mean_power_contrast_normalized_by_treatment_instruction_rate",
        "formula": "(treatment_mean_power_w - reference_mean_power_w) / treatment_scalar_instruction_rate_s * 1e12",
        "equal_work_energy_difference": False, "same_duration_required": False,
        "treatment_duration_s": result.get("duration_s"), "reference_duration_s": ref_phase.get("duration_s"),
        "treatment_power_w": result.get("board_power_w"), "reference_power_w": reference_power, "power_delta_w": contrast,
        "treatment_counted_instructions": counted, "reference_counted_loop_slots": slots,
        "treatment_completed_launches": bench.get("kernel_launches"), "reference_completed_launches": reference.get("kernel_launches"),
        "reference_actual_sfu_instructions": reference.get("sfu_instructions"),
        "reference_kernel_implementation_version": reference.get("kernel_implementation_version"),
        "reference_kernel_resources": reference.get("kernel_resources"),
        "reference_auxiliary_work": reference.get("auxiliary_work"),
        "reference_count_source": reference.get("block_completion_count_source"),
        "signed_observation": True, "hardware_attribution_proven": False,
        "uncertainty_scope": "repeat uncertainty is reported separately; telemetry bias and comparator-model error are not included",
        "treatment_scalar_instruction_rate_s": rate, "reference_loop_slots_s": slots_rate,
        "reference_to_treatment_issue_rate_ratio": slots_rate / rate if slots_rate is not None and rate else None,
        "reference_to_treatment_count_ratio": slots / counted if slots is not None and counted else None,
        "equal_selected_loop_slot_counts": slots == counted,
        "epilogue_logical_bytes_per_treatment_instruction":
            4 / (bench["iterations_per_launch"] * bench["sfu_chains"]) if count_ok else None,
        "epilogue_scope": "one final4B hash store per lane/launch; requested logical output only, not observed physical memory traffic"}


# ---------------------------------------------------------------------------- measurement diagnostics
def _ratio(a, b):
    return a / b if a is not None and b is not None and b > 0 else None


def _denominator(result: Mapping) -> tuple:
    """(unit, energy-metric suffix, rate per s, selected count) of a trial's work denominator."""
    workload = result.get("workload")
    if workload in MEMORY_WORKLOADS:
        rate, count = finite(result.get("throughput_bytes_s")), finite(result.get("counted_measure_logical_bytes"))
        return ("logical bit", "pj_per_logical_bit", rate * 8 if rate is not None else None,
                count * 8 if count is not None else None)
    if workload in SFU_WORKLOADS or workload in TENSOR_WORKLOADS or workload in NONLINEAR_WORKLOADS:
        unit, suffix = (("scalar SFU instruction", "pj_per_instruction") if workload in SFU_WORKLOADS else
                        ("FLOP", "pj_per_flop") if workload in TENSOR_WORKLOADS else ("element", "pj_per_element"))
        return unit, suffix, finite(result.get("throughput_ops_s")), finite(result.get("counted_measure_operations"))
    return None, None, None, None


_OBJECTIVE_FIELDS = (("total", "total_", "board_power_w", "total_energy_j"),
                     ("operational_idle_increment", "operational_idle_increment_", "operational_idle_increment_power_w",
                      "operational_idle_increment_energy_j"),
                     ("paired_active_reference", "paired_active_reference_", "paired_active_reference_power_w",
                      "paired_active_reference_energy_j"))


def _objective(result: Mapping, name: str, prefix: str, power_field: str, energy_field: str, unit, suffix, rate,
               count, exact: bool) -> dict:
    eligible = (result.get("valid") is True and exact if name == "total"
                else result.get(name + "_eligible") is True)
    power, energy = finite(result.get(power_field)), finite(result.get(energy_field))
    metric = prefix + suffix if suffix else None
    reported = finite(result.get(metric)) if metric else None
    rebuilt = _ratio(energy, count) if exact else _ratio(power, rate)
    rebuilt = rebuilt * 1e12 if rebuilt is not None else None
    return {"metric": metric, "unit": "pJ/" + unit if unit else None, "reported_value": reported,
            "reconstructed_value": rebuilt,
            "reconstruction_difference": reported - rebuilt if None not in (reported, rebuilt) else None,
            "power_w": power, "energy_j": energy, "eligible": eligible,
            "scope": "whole-device total" if name == "total" else
                     "whole-device operational contrast; physical component energy is not isolated"}


def _aliases(result: Mapping, bench: Mapping, unit, suffix) -> dict:
    workload = result.get("workload")
    if workload in MEMORY_WORKLOADS:
        ops, nbytes = finite(result.get("counted_measure_operations")), finite(result.get("counted_measure_logical_bytes"))
        per_op = _ratio(nbytes * 8 if nbytes is not None else None, ops)
        return {"pj_per_logical_byte": {"canonical_metric": "operational_idle_increment_pj_per_logical_bit", "value_multiplier": 8, "unit": "pJ/logical byte"},
                "total_pj_per_logical_byte": {"canonical_metric": "total_pj_per_logical_bit", "value_multiplier": 8, "unit": "pJ/logical byte"},
                "pj_per_op": {"canonical_metric": "operational_idle_increment_pj_per_logical_bit", "value_multiplier": per_op,
                              "unit": bench.get("operation_unit", "pJ/reported memory operation")}}
    if workload in TENSOR_WORKLOADS or workload in NONLINEAR_WORKLOADS:
        return {"pj_per_op": {"canonical_metric": "operational_idle_increment_" + suffix, "value_multiplier": 1, "unit": "pJ/" + unit},
                "total_pj_per_op": {"canonical_metric": "total_" + suffix, "value_multiplier": 1, "unit": "pJ/" + unit}}
    return {}


def measurement_diagnostics(result: Mapping, bench: Mapping, epochs: list) -> dict[str, Any]:
    """Each objective's reported value beside its reconstruction from energy and count (or power
    and rate), the scope factors between objectives, power shares, telemetry and timing."""
    memory, tensor = result.get("workload") in MEMORY_WORKLOADS, result.get("workload") in TENSOR_WORKLOADS
    unit, suffix, rate, count = _denominator(result)
    duration = finite(result.get("duration_s"))
    exact = result.get("count_energy_time_alignment_exact") is True
    objectives = {name: _objective(result, name, prefix, pf, ef, unit, suffix, rate, count, exact)
                  for name, prefix, pf, ef in _OBJECTIVE_FIELDS}
    board, idle = finite(result.get("board_power_w")), finite(result.get("idle_power_w"))
    reference, paired = finite(result.get("active_reference_power_w")), finite(result.get("paired_active_reference_power_w"))
    incremental = finite(result.get("operational_idle_increment_power_w"))
    integral, counter = finite(result.get("integrated_power_energy_j")), finite(result.get("energy_counter_j"))
    durations = [e["end_s"] - e["start_s"] for e in epochs]
    span = epochs[-1]["end_s"] - epochs[0]["start_s"] if epochs else None
    readbacks = [finite(e.get("counter_readback_ns")) for e in epochs]
    readback_s = sum(readbacks) / 1e9 if readbacks and all(v is not None and v >= 0 for v in readbacks) else None
    ops = finite(result.get("counted_measure_operations"))
    nbytes = finite(result.get("counted_measure_logical_bytes"))
    return {
        "schema_version": 1,
        "denominator": {"unit": unit, "measured_count": count if exact else None, "selected_epoch_count": count,
                        "rate_per_s": rate, "aligned_window_s": duration, "exact_matching_window": exact,
                        "kind": "same-window counted work" if exact else "stationary whole-run throughput estimate; no exact energy-window work count"},
        "objectives": objectives,
        "unit_conventions": {"bits_per_byte": 8 if memory else None, "flops_per_fma": 2 if tensor else None,
                             "flop_convention": result.get("flop_count_convention"),
                             "reported_operation_unit": bench.get("operation_unit"),
                             "logical_bits_per_reported_memory_operation": _ratio(nbytes * 8 if nbytes is not None else None, ops) if memory else None,
                             "logical_byte_scope": "requested read payload plus requested write payload for copy; not physical cache-sector or DRAM traffic" if memory else None,
                             "aliases": _aliases(result, bench, unit, suffix)},
        "scope_factors": {"total_over_idle_increment": _ratio(board, incremental),
                          "total_over_paired_reference": _ratio(board, paired),
                          "idle_increment_eligible": result.get("operational_idle_increment_eligible") is True,
                          "paired_reference_eligible": result.get("paired_active_reference_eligible") is True,
                          "interpretation": "Numerical operational scope ratios only; ineligible contrasts and component literature must not be silently substituted."},
        "power_contributions": {"total_w": board, "idle_w": idle, "idle_fraction": _ratio(idle, board),
                                "paired_reference_w": reference, "paired_reference_fraction": _ratio(reference, board),
                                "idle_increment_w": incremental, "paired_contrast_w": paired},
        "telemetry_crosscheck": {"energy_source": result.get("energy_source"), "counter_energy_j": counter,
                                 "integrated_power_energy_j": integral, "counter_over_integrated": _ratio(counter, integral),
                                 "disagreement_fraction": abs(counter - integral) / integral if counter is not None and integral is not None and integral > 0 else None},
        "throughput_crosscheck": {"unit": unit + "/s" if unit else None, "sustained_rate_per_s": rate,
                                  "profiler_replay_rate_per_s": None, "profiler_replay_count": None,
                                  "profiler_replay_summed_kernel_duration_s": None, "profiler_over_sustained_rate": None,
                                  "profiler_target_verified": result.get("target_verified") is True, "same_energy_run": False,
                                  "note": "Profiler replay uses a different run and summed kernel duration. Rate disagreement can motivate timing/traffic review but does not prove host overhead, permit energy rescaling or supply same-window physical traffic."},
        "execution": {"kernel_resources": bench.get("kernel_resources"), "sfu_contract": result.get("sfu_contract"),
                      "sfu_reference_delta": result.get("sfu_reference_delta_diagnostics"),
                      **{k: bench.get(k) for k in ("auxiliary_work", "execution_diagnostics")},
                      "implementation_version": bench.get("kernel_implementation_version"),
                      **{k: bench.get(k) for k in ("memory_accesses_per_thread_iteration", "memory_read_checksum_scope",
                                                   "memory_read_validation", "grid_mode", "input_elements",
                                                   "block_completion_count_source", "active_sm_ids",
                                                   "active_sm_distribution_status", "sm_distribution_scope")},
                      "saturation_status": "CUDA occupancy bounds and grid size do not establish achieved utilization or hardware saturation"},
        "timing": {"host_duration_s": finite(bench.get("host_duration_s")), "event_duration_s": finite(bench.get("duration_s")),
                   "event_duration_scope": bench.get("duration_scope", "CUDA experiment window; summed kernel busy time is not established"),
                   "mean_batch_experiment_duration_s": finite(bench.get("mean_batch_duration_s")),
                   "complete_epochs": len(epochs), "complete_epoch_span_s": span,
                   "summed_epoch_duration_s": sum(durations) if durations else None,
                   "inter_epoch_gap_s": max(0.0, span - sum(durations)) if span is not None else None,
                   "counter_readback_s": readback_s, "counter_readback_fraction": _ratio(readback_s, duration),
                   "kernel_busy_time_s": None,
                   "note": "Host synchronization, launch and readback gaps remain in sustained experiment energy and throughput. CUDA event-window rate is not a kernel-busy rate; NCU replay is a separate run."},
        "quality": {"valid": result.get("valid") is True, "issues": result.get("issues", []),
                    "baseline_valid": result.get("baseline_valid") is True, "baseline_issues": result.get("baseline_issues", []),
                    "target_verified": result.get("target_verified") is True},
    }


def rail_sources_of(phase_selected) -> list:
    """Sorted memory-power sources of the samples that report a memory power."""
    return sorted({s.get("memory_power_source") for samples in phase_selected
                   for s in samples if s.get("memory_power_w") is not None and s.get("memory_power_source")})


# ---------------------------------------------------------------------------- the whole trial
def complete_trial(record: Mapping, result: dict, trim_s: float, binding: list, rail_sources: list) -> dict:
    """Add the reporting fields to ``result`` (in place; also returned).

    ``binding``: binding_samples of the measure phase's selected samples (the aligned window);
    ``rail_sources``: the memory-power sources seen in the selected samples of idle_pre, measure,
    idle_post and active_control (rail_sources_of)."""
    from .contracts import sfu_count_issues
    bench = record.get("benchmark") or record.get("result") or {}
    device = record.get("device") or {}
    config = result.get("config") or {}
    workload = record.get("workload")
    phases_rec = record.get("phases") or {}
    if isinstance(phases_rec, list):
        phases_rec = {p["name"]: p for p in phases_rec if isinstance(p, dict) and "name" in p}
    epochs = kept_epochs(bench, phases_rec.get("measure"), trim_s) if result.get("complete_measure_epochs") else []
    result.update(_profiler_state(record, bench, config, result))
    result.update(_passthrough(record, bench, device))
    result.update(_statements(record, bench, result, epochs))
    result["validation_binding"] = _validation_binding(record, bench, config, binding)
    result["memory_rail_sources"] = rail_sources
    if workload == "l2_latency":
        result["latency_diagnostics"] = dict(bench)
    if phases_rec.get("active_control"):
        result["control_subtraction_note"] = _CONTROL_NOTE
    if workload in SFU_WORKLOADS:
        result.update(sfu_reference_delta_positive_optimum_eligible=False,
                      sfu_instruction_count_convention="one approximate PTX primitive application per active scalar lane; not warp instructions, FLOPs or complete-function elements",
                      sfu_reference_delta_estimator="mean_power_contrast_normalized_by_treatment_instruction_rate",
                      sfu_hardware_attribution_proven=False)
        if phases_rec.get("active_reference"):
            _sfu_diagnostics(record, bench, result, not sfu_count_issues(bench, workload))
    result["energy_peak_population_eligible"] = peak_population_eligible(result)
    diagnostics = _record_native().measurement_diagnostics(result, bench, epochs, MEMORY_WORKLOADS, TENSOR_WORKLOADS,
                                                           SFU_WORKLOADS, NONLINEAR_WORKLOADS, sum)
    diagnostics["memory_access_geometry"] = result["memory_access_geometry"]
    diagnostics["memory_coalescing"] = result["memory_coalescing"]
    result["measurement_diagnostics"] = diagnostics
    return result


# ---------------------------------------------------------------------------- groups
def _median(values):
    import statistics
    numbers = [v for v in (finite(x) for x in values) if v is not None]
    return statistics.median(numbers) if numbers else None


def group_coalescing(valid: list) -> dict | None:
    """The repeats' coalescing records as one: every repeat must pass for energy eligibility,
    ratios and efficiencies are medians (analysis.py:1379-1397)."""
    rows = [t.get("memory_coalescing") for t in valid if isinstance(t.get("memory_coalescing"), dict)]
    if not rows:
        return None
    statuses = {r.get("status") for r in rows}
    every = len(rows) == len(valid)
    out = dict(rows[0])
    out.update(status="fail" if "fail" in statuses else "pass" if statuses == {"pass"} else "inconclusive",
               energy_eligible=every and all(r.get("energy_eligible") is True for r in rows),
               profile_binding_verified=every and all(r.get("profile_binding_verified") is True for r in rows),
               bound_sector_ratio_failure=any(r.get("status") == "fail" and r.get("profile_binding_verified") is True for r in rows),
               reasons=sorted({reason for r in rows for reason in r.get("reasons", [])}),
               aggregation="Median of valid repeat replay ratios/efficiencies; all repeats must pass for energy eligibility. These replay values never replace energy-run logical work.")
    for field in ("requested_sector_efficiency_fraction", "observed_sector_bytes_per_logical_read_byte",
                  "observed_sector_efficiency_fraction", "observed_sector_efficiency_pct"):
        out[field] = _median(r.get(field) for r in rows)
    for field in ("counter_name", "counter_scope"):
        values = {r.get(field) for r in rows}
        out[field] = next(iter(values)) if len(values) == 1 else None
    return out


def _median_of(numbers: list) -> float:
    """statistics.median of a non-empty list of floats."""
    numbers.sort()
    n = len(numbers)
    mid = n // 2
    return numbers[mid] if n % 2 else (numbers[mid - 1] + numbers[mid]) / 2


def _record_native():
    try:
        from . import _recordnative
    except ImportError as exc:
        from ._native import NativeError
        raise NativeError("the record assembly extension (_recordnative) is not built; run powermodeling_b200.build") from exc
    return _recordnative


def _fold(values: list):
    """Repeat diagnostics as one: dicts key by key, lists as their distinct items, flags all-true,
    numbers by their median, anything else as the first present value."""
    first = next((v for v in values if v is not None), None)
    kind = type(first)
    if kind is dict or isinstance(first, dict):
        keys = dict.fromkeys(k for v in values if isinstance(v, dict) for k in v)
        return {k: _fold([v.get(k) if isinstance(v, dict) else None for v in values]) for k in keys}
    if kind is list or isinstance(first, list):
        import json
        return list({json.dumps(item, sort_keys=True): item for v in values if isinstance(v, list) for item in v}.values())
    if kind is bool:
        return all(v is True for v in values)
    if kind is str or first is None:
        return first
    numbers = []
    for v in values:
        t = type(v)
        if t is float or t is int:
            if math.isfinite(v):
                numbers.append(float(v))
        elif isinstance(v, (int, float)) and not isinstance(v, bool):
            f = finite(v)
            if f is not None:
                numbers.append(f)
    return _median_of(numbers) if numbers else first


def group_diagnostics(valid: list, group: Mapping) -> dict:
    """The group's measurement diagnostics: each numeric field the median of its repeats'
    (analysis.py:567-595)."""
    if not valid:
        return {"schema_version": 1, "valid_repeats": 0, "aggregation": "no valid repeat diagnostics"}
    folded = _record_native().fold([t["measurement_diagnostics"] for t in valid], _fold)
    folded.update(schema_version=1, valid_repeats=len(valid),
                  aggregation="Each numeric diagnostic is the median of valid repeat diagnostics; reconstructed energy/work and scope factors are medians of per-repeat ratios, not ratios of separately aggregated powers/counts.")
    for objective, flag in (("operational_idle_increment", "idle_increment_eligible"),
                            ("paired_active_reference", "paired_reference_eligible")):
        eligible = group.get(objective + "_eligible") is True
        folded["objectives"][objective]["eligible"] = eligible
        folded["scope_factors"][flag] = eligible
    return folded


def complete_group(group: dict, first: Mapping, valid: list, min_repeats: int) -> dict:
    """Add the group fields that follow from its repeats' reporting fields (in place; also returned).
    ``first``: the group's first trial (valid or not); ``valid``: its valid, non-duplicate repeats."""
    group.update(memory_access_geometry=first.get("memory_access_geometry"), memory_coalescing=group_coalescing(valid),
                 memory_coalescing_energy_eligible=(bool(valid) and all(t.get("memory_coalescing_energy_eligible") is True for t in valid))
                 if first.get("memory_coalescing") is not None else None,
                 kernel_resources=first.get("kernel_resources"), execution_diagnostics=first.get("execution_diagnostics"),
                 memory_accesses_per_thread_iteration=first.get("memory_accesses_per_thread_iteration"),
                 target_verified=bool(valid) and all(t["target_verified"] for t in valid),
                 verified_selection_eligible=bool(valid) and all(t["verified_selection_eligible"] for t in valid))
    statuses = {t["ncu_status"] for t in valid}
    group["ncu_status"] = ("fail" if "fail" in statuses else "pass" if statuses == {"pass"} else
                           "unprofiled" if statuses == {"unprofiled"} else "inconclusive")
    if group["workload"] in SFU_WORKLOADS:
        counterbalanced = group["paired_reference_counterbalanced"]
        group["sfu_reference_delta_measurement_valid"] = (
            bool(valid) and all(t.get("sfu_reference_delta_measurement_valid") is True for t in valid) and counterbalanced)
        interval = group["ci95"].get("sfu_reference_delta_pj_per_instruction")
        group["ci95"]["paired_active_reference_pj_per_instruction"] = interval
        crosses = interval[0] <= 0 <= interval[1] if interval else None
        group["sfu_reference_delta_ci_crosses_zero"] = crosses
        group["sfu_reference_delta_positive_optimum_eligible"] = (
            group["sfu_reference_delta_measurement_valid"] and group["verified_selection_eligible"]
            and len(valid) >= min_repeats and bool(interval) and interval[0] > 0)
        group["sfu_hardware_attribution_proven"] = False
        group["sfu_reference_delta_estimator"] = "mean_power_contrast_normalized_by_treatment_instruction_rate"
        group["sfu_reference_delta_issues"] = sorted({i for t in valid for i in t.get("sfu_reference_delta_issues", [])}
                                                     | (set() if counterbalanced else {"paired_orders_not_counterbalanced"}))
        group["sfu_reference_delta_uncertainty"] = {
            "ci95_pj_per_instruction": interval, "ci_crosses_zero": crosses,
            "method": "percentile bootstrap of repeat paired-contrast medians",
            "scope": "repeat uncertainty only; telemetry bias, comparator model error and physical attribution uncertainty are not bounded",
            "signed_observation_retained": True}
    group["ncu_target_suitability"] = group["target_verified"]
    group["ncu_utilization_status"] = ("diagnostic_only" if valid and all(t["ncu_utilization_status"] == "diagnostic_only" for t in valid)
                                       else "inconclusive")
    diagnostics = group_diagnostics(valid, group)
    group["measurement_diagnostics"] = diagnostics
    group["energy_peak_population_eligible"] = peak_population_eligible(group)
    diagnostics["memory_access_geometry"] = group["memory_access_geometry"]
    diagnostics["memory_coalescing"] = group["memory_coalescing"]
    if group["workload"] in SFU_WORKLOADS:
        group["sfu_reference_delta_diagnostics"] = (diagnostics.get("execution") or {}).get("sfu_reference_delta")
    return group
