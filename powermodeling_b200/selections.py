"""Best conditions, energy optima and Pareto frontiers over a summary's groups.

The caller-side consumer of the group medians and intervals: which measured
condition is the most energy-efficient in each comparable stratum, under a
throughput bar (the reference's summarize sections ``within_clock_best`` ...
``exploratory_single_geometry_overall_energy_optima``, analysis.py:1104-1376,
with the eligibility rules of evaluation.py:67-103 and hbm_bandwidth.py:128-143).

The design here: a workload family maps to the rate and energy fields it is
judged on (``rate_field``, ``energy_field``, ``selection_field``); a section
is a filter of the groups by eligibility predicates, a bucketing by a stratum
key (``clock_stratum``) and a choice within each bucket.  Record keys,
strings and ordering are the reference's, since summary.json carries them.
"""
from __future__ import annotations

import json
import math
from typing import Any, Mapping

TENSOR = {"tensor", "fp16_tensor", "tensor_fp16", "gemm"}
MEMORY = {"l1", "l2", "hbm"}
SFU = {"sfu_ex2", "sfu_lg2", "sfu_rcp", "sfu_rsqrt", "sfu_sqrt", "sfu_tanh"}
NONLINEAR = {"exp", "tanh", "silu", "rmsnorm", "softmax"}
COMPUTE = TENSOR | NONLINEAR | SFU
ENERGY = COMPUTE | MEMORY
ROLES = ("energy_characterization", "legacy_unspecified")
HBM_DEFAULT_FRACTION = 0.80


def _number(value) -> float | None:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
        return None
    return float(value)


def rate_field(workload: str) -> str:
    """The throughput a workload is judged on (SFU instructions, operations, or logical bytes)."""
    return "throughput_sfu_instructions_s" if workload in SFU else "throughput_ops_s" if workload in COMPUTE \
        else "throughput_bytes_s"


def energy_field(workload: str, prefix: str) -> str:
    unit = ("pj_per_instruction" if workload in SFU else "pj_per_element" if workload in NONLINEAR
            else "pj_per_flop" if workload in TENSOR else "pj_per_logical_bit")
    return prefix + unit


def selection_field(workload: str, total_energy: bool) -> str:
    """The metric a best-condition selection minimises (the legacy per-op / per-byte names)."""
    if workload in SFU:
        return "sfu_reference_delta_pj_per_instruction"
    unit = "pj_per_element" if workload in NONLINEAR else "pj_per_op" if workload in TENSOR else "pj_per_logical_byte"
    return ("total_" if total_energy else "") + unit


# ---------------------------------------------------------------------------- memory read geometry
def read_geometry(benchmark: Mapping | None, workload: str, config: Mapping | None = None) -> dict[str, Any]:
    """Whether a scalar read's declared geometry keeps every warp on whole 32-byte sectors
    (memory.py:19-107): unit word stride, sector-aligned offset and region, whole warps.
    A declaration check only; observed traffic needs profiler counters."""
    benchmark, config = benchmark or {}, config or {}
    get = lambda key, default=None: benchmark[key] if key in benchmark else config.get(key, default)  # noqa: E731
    applicable = workload in MEMORY and get("access", "read") == "read"
    out: dict[str, Any] = {
        "applicable": applicable, "status": "inconclusive", "energy_eligible": False,
        "reasons": [], "word_bytes": 4, "sector_bytes": 32,
        "expected_sector_efficiency_fraction": 1.0 if applicable else None,
        "requested_sector_efficiency_fraction": None,
        "requested_sector_efficiency_scope": "first full warp scalar read at the declared region base, without wrapping or duplicate addresses; observed counters are required",
        "effective_region_bytes": None, "region_source": None,
        "base_alignment_scope": "CUDA allocation base plus offset; each L1 CTA adds its slice size; sector alignment does not require 128-byte alignment",
    }
    if not applicable:
        out["reasons"] = ["coalesced_read_energy_not_applicable"]
        return out
    failures, unknown = set(), set()

    def whole(key, default=None, minimum=0):
        value = get(key, default)
        number = _number(value)
        if value is None:
            unknown.add("missing_geometry:" + key)
        elif number is None or number < minimum or not number.is_integer():
            failures.add("invalid_geometry:" + key)
        else:
            return int(value)
        return None

    stride, offset = whole("stride_elements", 1, 1), whole("offset_bytes", 0)
    threads, working_set = whole("threads", minimum=1), whole("working_set_bytes", minimum=4)
    lane_bytes = None if stride is None else stride * 4
    out.update(stride_elements=stride, stride_words=stride, lane_stride_bytes=lane_bytes, offset_bytes=offset,
               threads=threads)
    for key, expected in (("memory_word_bytes", 4), ("stride_words", stride), ("lane_stride_bytes", lane_bytes)):
        if key in benchmark or key in config:
            declared = _number(get(key))
            if declared is None or declared <= 0 or not declared.is_integer():
                failures.add("invalid_geometry:" + key)
            elif expected is not None and declared != expected:
                failures.add("inconsistent_word_stride_metadata:" + key)
    for reason, broken in (("nonunit_word_stride", stride is not None and stride != 1),
                           ("offset_not_sector_aligned", offset is not None and offset % 32),
                           ("threads_not_complete_supported_warps",
                            threads is not None and (threads < 32 or threads > 1024 or threads % 32)),
                           ("working_set_not_word_aligned", working_set is not None and working_set % 4)):
        if broken:
            failures.add(reason)
    region, out["region_source"] = working_set, "working_set_bytes"
    if workload == "l1":
        blocks = whole("blocks", minimum=1)
        derived = working_set // 4 // blocks * 4 if working_set is not None and blocks else None
        if get("l1_bytes_per_block") is not None:
            region, out["region_source"] = whole("l1_bytes_per_block", minimum=4), "l1_bytes_per_block"
            if derived is not None and region is not None and region != derived:
                failures.add("l1_slice_disagrees_with_working_set_and_blocks")
        else:
            region, out["region_source"] = derived, "floor(working_set_words/blocks)*4"
    out["effective_region_bytes"] = region
    if region is None:
        unknown.add("effective_region_unknown")
    elif region < 128:
        failures.add("region_smaller_than_full_warp_payload")
    elif region % 32:
        failures.add("region_not_sector_aligned")
    if stride is not None and offset is not None:
        touched = {(offset % 32 + lane * stride * 4) // 32 for lane in range(32)}
        out["requested_sector_efficiency_fraction"] = 128 / (len(touched) * 32)
    out["reasons"] = sorted(failures | unknown)
    out["status"] = "fail" if failures else "inconclusive" if unknown else "pass"
    out["energy_eligible"] = out["status"] == "pass"
    return out


# ---------------------------------------------------------------------------- eligibility
def _contract(group: Mapping) -> Mapping:
    return group.get("experiment_contract") or {}


def _access(group: Mapping) -> str:
    return _contract(group).get("access", (group.get("config") or {}).get("access", "read"))


def role_eligible(group: Mapping) -> bool:
    """An energy-characterisation (or unlabelled) group, and not an HBM read bypassing .cg (evaluation.py:67-72)."""
    cache = _contract(group).get("read_cache_policy", (group.get("config") or {}).get("read_cache_policy", "cg"))
    hbm_uncached = group.get("workload") == "hbm" and _access(group) == "read" and cache != "cg"
    return group.get("experiment_role", "legacy_unspecified") in ROLES and not hbm_uncached


def _memory_read(group: Mapping) -> bool:
    return group.get("workload") in MEMORY and _contract(group).get(
        "access", group.get("config", {}).get("access", "read")) == "read"


def coalescing_eligible(group: Mapping) -> bool:
    """Memory reads need profiler-confirmed coalescing for every valid repeat (evaluation.py:80-81)."""
    return not _memory_read(group) or group.get("memory_coalescing_energy_eligible") is True


def peak_population_eligible(group: Mapping) -> bool:
    """May this group's rate define a throughput bar: strided or misaligned reads may not, and
    neither may a read whose sector ratio a bound profile failed (evaluation.py:84-103)."""
    if not role_eligible(group):
        return False
    if not _memory_read(group):
        return True
    geometry = group.get("memory_access_geometry")
    if not isinstance(geometry, dict):
        geometry = read_geometry({**group.get("config", {}), **_contract(group), **(group.get("resource_geometry") or {})},
                                 group.get("workload"))
    coalescing = group.get("memory_coalescing") or {}
    bound_failure = coalescing.get("bound_sector_ratio_failure") is True or (
        coalescing.get("status") == "fail" and coalescing.get("profile_binding_verified") is True)
    return geometry.get("energy_eligible") is True and not bound_failure


def meets_bar(group: Mapping, rate: str, peak, fraction: float) -> bool:
    """HBM passes on its own interface gate; every other workload at ``fraction`` of an observed peak."""
    if group.get("workload") == "hbm":
        return (group.get("hbm_bandwidth") or {}).get("eligible") is True
    value, bar = _number(group.get(rate)), _number(peak)
    return value is not None and bar is not None and bar > 0 and value >= fraction * bar


def bar_metadata(group: Mapping, fraction: float) -> dict[str, Any]:
    hbm = group.get("workload") == "hbm"
    evidence = group.get("hbm_bandwidth") or {}
    return {"throughput_threshold_basis": "clock_specific_hbm_theoretical_bandwidth" if hbm else "observed_peak",
            "throughput_threshold_fraction": evidence.get("minimum_fraction", HBM_DEFAULT_FRACTION) if hbm else fraction,
            "observed_peak_threshold_fraction": fraction, "hbm_bandwidth": group.get("hbm_bandwidth")}


def clock_stratum(group: Mapping, cross_clock: bool) -> dict[str, Any]:
    """The conditions a comparison holds fixed: device, workload contract, strata, and, within a
    clock, the requested clocks (analysis.py:1104-1119)."""
    config = group["config"]
    key = {"gpu_uuid": group["gpu_uuid"], "workload": group["workload"],
           "experiment_role": group.get("experiment_role", "legacy_unspecified"),
           "experiment_contract": group.get("experiment_contract"),
           "benchmark_sha256": group.get("benchmark_sha256"), "measurement_stratum": group.get("measurement_stratum"),
           "treatment_design_stratum": group.get("treatment_design_stratum"),
           "access": config.get("access", "read") if group["workload"] in MEMORY else None}
    if group["workload"] in NONLINEAR:
        key["nonlinear_contract"] = group.get("nonlinear_contract")
    if group["workload"] in SFU:
        key["sfu_contract"] = group.get("sfu_contract")
    if not cross_clock:
        key.update(graphics_clock_mhz=config.get("graphics_clock_mhz") or group.get("graphics_clock_mhz"),
                   memory_clock_mhz=config.get("memory_clock_mhz") or group.get("memory_clock_mhz"),
                   clock_comparison_controlled=group["clock_comparison_controlled"])
    return key


def _key(stratum: Mapping) -> str:
    return json.dumps(stratum, sort_keys=True)


# Within ``stratum_memo()``, each group's stratum and key are computed once per
# comparison scope (the summary evaluates a dozen sections over the same groups).
_MEMO: dict | None = None


class stratum_memo:
    """Context in which stratum_of caches by group identity (the groups must outlive it)."""

    def __enter__(self):
        global _MEMO
        self.outer, _MEMO = _MEMO, {}
        return self

    def __exit__(self, *exc):
        global _MEMO
        _MEMO = self.outer


def stratum_of(group: Mapping, cross_clock: bool) -> tuple[str, dict]:
    """(key string, stratum) of clock_stratum(group, cross_clock)."""
    if _MEMO is None:
        stratum = clock_stratum(group, cross_clock)
        return _key(stratum), stratum
    slot = (id(group), cross_clock)
    hit = _MEMO.get(slot)
    if hit is None:
        stratum = clock_stratum(group, cross_clock)
        hit = _MEMO[slot] = (_key(stratum), stratum)
    return hit


def _bucket(items, key_of) -> list[tuple[str, list]]:
    buckets: dict[str, list] = {}
    for item in items:
        buckets.setdefault(key_of(item), []).append(item)
    return sorted(buckets.items(), key=lambda kv: kv[0])


# ---------------------------------------------------------------------------- best conditions
def _selectable(group: Mapping, min_repeats: int, verified_only: bool, total_energy: bool, exploratory_only: bool) -> bool:
    if not (role_eligible(group) and coalescing_eligible(group)) or group["workload"] not in ENERGY:
        return False
    if group["valid_repeats"] < min_repeats or exploratory_only == group["clock_comparison_controlled"]:
        return False
    sfu = group["workload"] in SFU
    if sfu and (total_energy or not group.get("sfu_reference_delta_positive_optimum_eligible")):
        return False
    if verified_only and not group["verified_selection_eligible"]:
        return False
    if not (total_energy or sfu or group.get("operational_idle_increment_eligible")):
        return False
    return (group.get(selection_field(group["workload"], total_energy)) is not None
            and group.get(rate_field(group["workload"])) is not None)


def best_conditions(groups: list, fraction: float, min_repeats: int, cross_clock: bool, verified_only: bool = False,
                    total_energy: bool = False, exploratory_only: bool = False) -> list[dict[str, Any]]:
    """Per stratum, the group with the lowest energy metric among those at ``fraction`` of the
    stratum's peak rate (ties: the faster); the peak of a verified-only selection is the whole
    valid sweep's, so an incomplete verified subset cannot lower the bar."""
    chosen = [g for g in groups if _selectable(g, min_repeats, verified_only, total_energy, exploratory_only)]
    out = []
    for key, candidates in _bucket(chosen, lambda g: stratum_of(g, cross_clock)[0]):
        first = candidates[0]
        metric, rate = selection_field(first["workload"], total_energy), rate_field(first["workload"])
        stratum = json.loads(key)
        candidate_max = max(g[rate] for g in candidates)
        population = [g[rate] for g in groups
                      if g["workload"] == first["workload"] and peak_population_eligible(g)
                      and g["gpu_uuid"] == first["gpu_uuid"] and g["valid_repeats"] >= min_repeats
                      and g["clock_comparison_controlled"] == first["clock_comparison_controlled"]
                      and stratum_of(g, cross_clock)[1] == stratum and g.get(rate) is not None]
        sweep_max = max(population) if population else candidate_max
        bar = sweep_max if verified_only else candidate_max
        passing = [g for g in candidates if meets_bar(g, rate, bar, fraction)]
        if not passing:
            continue
        best = min(passing, key=lambda g: (g[metric], -g[rate]))
        out.append({"stratum": json.loads(key), "best_group_id": best["group_id"], "config": best["config"],
                    "metric": metric, "metric_value": best[metric], "metric_ci95": best["ci95"].get(metric),
                    "throughput": best[rate], "observed_max_throughput": bar,
                    "throughput_fraction_of_observed_max": best[rate] / bar if bar else None,
                    **bar_metadata(best, fraction), "eligible_groups": len(passing),
                    "target_verified": best["target_verified"], "valid_repeats": best["valid_repeats"],
                    "clock_comparison_controlled": best["clock_comparison_controlled"],
                    "observation_scope": "uncontrolled-clock exploratory" if exploratory_only else "requested fixed-clock comparison",
                    "observed_max_throughput_all_valid_groups": sweep_max,
                    "verified_peak_coverage_fraction": candidate_max / sweep_max if verified_only and sweep_max > 0 else None,
                    "meets_threshold_vs_all_valid_groups": meets_bar(best, rate, sweep_max, fraction),
                    "selection_scope": "best measured among tested configurations; sweep completeness and physical target attribution are not implied"})
    return out


# ---------------------------------------------------------------------------- Pareto, coverage, controls
def _controlled_population(group: Mapping, min_repeats: int) -> bool:
    return (peak_population_eligible(group) and group["workload"] in ENERGY and group["valid_repeats"] >= min_repeats
            and group["clock_comparison_controlled"])


def verification_coverage(groups: list, fraction: float, min_repeats: int, cross_clock: bool) -> list[dict[str, Any]]:
    """Per stratum, how much of the valid sweep's peak the profiler-verified groups reach."""
    valid = [g for g in groups if _controlled_population(g, min_repeats) and (g.get(rate_field(g["workload"])) or 0) > 0]
    out = []
    for key, candidates in _bucket(valid, lambda g: stratum_of(g, cross_clock)[0]):
        rate = rate_field(candidates[0]["workload"])
        peak = max(g[rate] for g in candidates)
        verified = [g for g in candidates if g["verified_selection_eligible"]]
        verified_peak = max(g[rate] for g in verified) if verified else None
        high = [g for g in verified if meets_bar(g, rate, peak, fraction)]
        status = ("eligible_verified_conditions_available" if high else
                  "no_verified_condition_reaches_hbm_theoretical_bandwidth_threshold" if candidates[0]["workload"] == "hbm"
                  else "no_verified_condition_reaches_complete_sweep_throughput_threshold")
        out.append({"stratum": json.loads(key), "scope": "cross_clock" if cross_clock else "within_clock",
                    "observed_max_throughput_all_valid_groups": peak,
                    "observed_max_throughput_verified_groups": verified_peak,
                    "verified_peak_coverage_fraction": verified_peak / peak if verified_peak is not None else 0,
                    **bar_metadata(candidates[0], fraction), "valid_groups": len(candidates),
                    "verified_groups": len(verified), "verified_high_throughput_groups": len(high),
                    "selection_status": status,
                    "unverified_or_failed_peak_group_ids": [g["group_id"] for g in candidates
                                                            if g[rate] == peak and not g["verified_selection_eligible"]]})
    return out


def pareto_frontiers(groups: list, min_repeats: int, cross_clock: bool) -> list[dict[str, Any]]:
    """Per stratum, the groups no other group beats on both rate (higher) and board power (lower)."""
    valid = [g for g in groups
             if role_eligible(g) and coalescing_eligible(g) and g["workload"] in ENERGY and g["valid_repeats"] >= min_repeats
             and g["clock_comparison_controlled"] and g.get("board_power_w") is not None
             and g.get(rate_field(g["workload"])) is not None]
    out = []
    for key, candidates in _bucket(valid, lambda g: stratum_of(g, cross_clock)[0]):
        rate = rate_field(candidates[0]["workload"])

        def dominated(g):
            return any(o[rate] >= g[rate] and o["board_power_w"] <= g["board_power_w"]
                       and (o[rate] > g[rate] or o["board_power_w"] < g["board_power_w"]) for o in candidates)

        front = sorted((g for g in candidates if not dominated(g)), key=lambda g: (g[rate], g["board_power_w"]))
        out.append({"stratum": json.loads(key), "scope": "cross_clock" if cross_clock else "within_clock",
                    "objectives": {"maximize": rate, "minimize": "board_power_w"},
                    "candidate_groups": len(candidates), "frontier": [
                        {"group_id": g["group_id"], "config": g["config"], "throughput": g[rate],
                         "board_power_w": g["board_power_w"], "incremental_power_w": g["incremental_power_w"],
                         "target_verified": g["target_verified"], "valid_repeats": g["valid_repeats"],
                         "clock_comparison_controlled": g["clock_comparison_controlled"]} for g in front],
                    "note": "Pareto dominance uses repeat medians; overlapping uncertainty intervals may change ordering."})
    return out


CONTROL_MATCH = ("graphics_clock_mhz", "memory_clock_mhz", "blocks", "threads", "sm_ids")


def control_associations(groups: list, min_repeats: int) -> list[dict[str, Any]]:
    """Each energy group's active-control groups on the same device, strata, clocks and launch geometry."""
    controls = [g for g in groups if g["workload"] == "control" and g["valid_repeats"] >= min_repeats]
    strata = ("benchmark_sha256", "measurement_stratum", "treatment_design_stratum")
    out = []
    for g in groups:
        if g["workload"] not in ENERGY or g["valid_repeats"] < min_repeats:
            continue
        found = [c for c in controls if c["gpu_uuid"] == g["gpu_uuid"]
                 and c.get("experiment_role", "legacy_unspecified") == g.get("experiment_role", "legacy_unspecified")
                 and all(c.get(s) == g.get(s) for s in strata)
                 and all(c["config"].get(f) == g["config"].get(f) for f in CONTROL_MATCH)]
        if found:
            out.append({"workload_group_id": g["group_id"], "control_groups": [
                {"group_id": c["group_id"], "board_power_w": c["board_power_w"],
                 "incremental_activation_power_w": c["incremental_power_w"]} for c in found],
                "matching_fields": ["gpu_uuid", "experiment_role", *strata, *CONTROL_MATCH],
                "note": "Descriptive activation controls only. Different instruction mixes prevent automatic component-energy subtraction."})
    return out


# ---------------------------------------------------------------------------- energy optima
OBJECTIVES = (("total", "total_", None),
              ("operational_idle_increment", "operational_idle_increment_", "operational_idle_increment_eligible"),
              ("paired_active_reference", "paired_active_reference_", "paired_active_reference_eligible"))


def _positive(value) -> float | None:
    number = _number(value)
    return number if number is not None and number > 0 else None


def energy_optima(groups: list, fraction: float, min_repeats: int, near_fraction: float, min_geometries: int = 2,
                  across_memory_domains: bool = False, single_geometry_exploratory: bool = False) -> list[dict[str, Any]]:
    """Each GPU's measured energy optimum per objective, among verified groups at ``fraction`` of
    their own clock's peak rate, where the clock has enough verified launch geometries to compare
    (analysis.py:1181-1298).  Every support point is a measured group; nothing is interpolated."""
    population = [g for g in groups if g["workload"] in ENERGY and peak_population_eligible(g)
                  and g["valid_repeats"] >= min_repeats and g["clock_comparison_controlled"]]
    own_clock = lambda g: stratum_of(g, False)[0]  # noqa: E731
    peaks: dict[str, float] = {}
    shapes: dict[str, set] = {}
    verified_shapes: dict[str, set] = {}
    for g in population:
        value = _positive(g.get(rate_field(g["workload"])))
        if value is None:
            continue
        clock = own_clock(g)
        peaks[clock] = max(peaks.get(clock, 0), value)
        geometry = g.get("resource_geometry") or {}
        if geometry and all(_positive(v) is not None for v in geometry.values()):
            signature = json.dumps(geometry, sort_keys=True)
            shapes.setdefault(clock, set()).add(signature)
            if g["verified_selection_eligible"]:
                verified_shapes.setdefault(clock, set()).add(signature)
    entries = []
    for g in population:
        if not g["verified_selection_eligible"]:
            continue
        rate, clock = rate_field(g["workload"]), own_clock(g)
        count = len(verified_shapes.get(clock, set()))
        if (count != 1) if single_geometry_exploratory else (count < min_geometries):
            continue
        if not meets_bar(g, rate, peaks.get(clock), fraction):
            continue
        for objective, prefix, eligibility in OBJECTIVES:
            if g["workload"] in SFU and (objective != "paired_active_reference"
                                         or not g.get("sfu_reference_delta_positive_optimum_eligible")):
                continue
            if eligibility and not g.get(eligibility):
                continue
            metric = energy_field(g["workload"], prefix)
            if _positive(g.get(metric)) is None:
                continue
            stratum = dict(stratum_of(g, True)[1])
            if not across_memory_domains:
                stratum["memory_clock_mhz"] = g["config"].get("memory_clock_mhz")
            stratum["objective"] = objective
            entries.append((_key(stratum), (g, metric, rate, peaks.get(clock))))
    buckets: dict[str, list] = {}
    for key, entry in entries:
        buckets.setdefault(key, []).append(entry)
    return [_optimum(key, buckets[key], shapes, verified_shapes, population, fraction, near_fraction, min_geometries,
                     across_memory_domains, single_geometry_exploratory) for key in sorted(buckets)]


_SCOPE_TEXT = {
    "selection": ("diagnostic single-geometry energy minimum; self-reference throughput ratio does not qualify high utilization",
                  "best observed eligible measured point; incomplete geometry, frequency or profiler coverage cannot establish the global hardware optimum"),
    "utilization": ("only one verified measured resource geometry; own-frequency peak ratio does not qualify utilization",
                    "at least min_geometries independently verified execution-resource geometries; throughput bar uses all valid observed groups and geometry count alone does not prove physical saturation"),
    "optimization": ("across measured graphics frequencies at one fixed memory domain",
                     "across measured graphics and memory frequency domains"),
}


def _optimum(key, candidates, shapes, verified_shapes, population, fraction, near_fraction, min_geometries, across,
             single) -> dict[str, Any]:
    group, metric, rate, clock_peak = min(candidates, key=lambda c: (c[0][c[1]], -c[0][c[2]], c[0]["group_id"]))
    best_ci = group["ci95"].get(metric)
    evidence = "single_geometry_reference_only" if single else "multiple_resource_geometries_compared"

    def counts(g) -> dict[str, int]:
        clock = stratum_of(g, False)[0]
        verified = len(verified_shapes.get(clock, set()))
        return {"own_clock_distinct_geometry_count": verified, "own_clock_verified_distinct_geometry_count": verified,
                "own_clock_observed_distinct_geometry_count": len(shapes.get(clock, set()))}

    def point(c) -> dict[str, Any]:
        g, m, r, peak = c
        return {"group_id": g["group_id"], "graphics_clock_mhz": g.get("graphics_clock_mhz"),
                "memory_clock_mhz": g.get("memory_clock_mhz"),
                "requested_graphics_clock_mhz": g["config"].get("graphics_clock_mhz"),
                "requested_memory_clock_mhz": g["config"].get("memory_clock_mhz"),
                "metric_value": g[m], "metric_ci95": g["ci95"].get(m), "throughput": g[r],
                "throughput_fraction_of_own_clock_observed_peak": g[r] / peak, **bar_metadata(g, fraction),
                "config": g["config"], "valid_repeats": g["valid_repeats"],
                "paired_reference_order_counts": g.get("paired_reference_order_counts"),
                "resource_geometry": g.get("resource_geometry"), **counts(g),
                "geometry_evidence_status": evidence, "saturation_proven": False}

    def points(chosen) -> list[dict[str, Any]]:
        return sorted((point(c) for c in chosen), key=lambda p: (p["requested_memory_clock_mhz"],
                                                                  p["requested_graphics_clock_mhz"], p["group_id"]))

    near = [c for c in candidates if c[0][metric] <= group[metric] * (1 + near_fraction)]
    overlap = [c for c in candidates if best_ci and c[0]["ci95"].get(metric)
               and c[0]["ci95"][metric][0] <= best_ci[1] and c[0]["ci95"][metric][1] >= best_ci[0]]
    stratum = json.loads(key)
    base = {k: v for k, v in stratum.items() if k not in ("objective", "memory_clock_mhz")}
    comparable = [p for p in population if stratum_of(p, True)[1] == base
                  and (across or p["config"].get("memory_clock_mhz") == stratum["memory_clock_mhz"])]
    observed = sorted({(p["config"].get("graphics_clock_mhz"), p["config"].get("memory_clock_mhz")) for p in comparable})
    eligible = sorted({(c[0]["config"].get("graphics_clock_mhz"), c[0]["config"].get("memory_clock_mhz")) for c in candidates})
    pairs = lambda items: [{"graphics_clock_mhz": gfx, "memory_clock_mhz": mem} for gfx, mem in items]  # noqa: E731
    return {"stratum": json.loads(key), "gpu_name": group.get("gpu_name"), "best_group_id": group["group_id"],
            "objective": stratum["objective"], "metric": metric, "metric_value": group[metric], "metric_ci95": best_ci,
            "config": group["config"], "winning_requested_graphics_clock_mhz": group["config"].get("graphics_clock_mhz"),
            "winning_requested_memory_clock_mhz": group["config"].get("memory_clock_mhz"),
            "winning_achieved_graphics_clock_mhz": group.get("graphics_clock_mhz"),
            "winning_achieved_memory_clock_mhz": group.get("memory_clock_mhz"),
            "throughput": group[rate], "own_clock_observed_max_throughput": clock_peak,
            "throughput_fraction_of_own_clock_observed_peak": group[rate] / clock_peak,
            **bar_metadata(group, fraction), "candidate_groups": len(candidates), **counts(group),
            "geometry_evidence_status": evidence, "min_geometries_required": min_geometries, "saturation_proven": False,
            "selection_status": "exploratory_single_geometry_only" if single else "geometry_comparison_qualified_best_observed",
            "observed_valid_frequency_pairs": pairs(observed), "eligible_frequency_pairs": pairs(eligible),
            "observed_frequency_pairs_without_eligible_candidate": pairs(sorted(set(observed) - set(eligible))),
            "selection_scope": _SCOPE_TEXT["selection"][0 if single else 1],
            "near_optimum_relative_tolerance": near_fraction,
            "near_optimum_support_points": points(near), "uncertainty_overlap_support_points": points(overlap),
            "all_eligible_support_points": points(candidates),
            "optimal_interval_kind": "discrete measured support points; unmeasured gaps and continuous intervals are not inferred",
            "optimization_scope": _SCOPE_TEXT["optimization"][1 if across else 0],
            "utilization_basis": _SCOPE_TEXT["utilization"][0 if single else 1],
            "energy_scope": "whole-device energy per counted logical bit, dense tensor FLOP or complete nonlinear output element; physical component energy is not isolated"}
