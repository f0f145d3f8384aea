"""Component evaluation of a summary: what each measured component shows, with
the evidence it lacks written out (the reference's ``evaluate``,
evaluation.py:436-640, and its helpers 24-435).

A component is one comparable stratum of groups (GPU, workload, binary,
measurement and treatment strata, experiment contract and role).  It is built
in stages, each a function of the component's groups and a shared context:

* ``_point``: one row per group: rates, energies per objective and their
  intervals, and per objective the reasons it cannot be a candidate, from the
  rule table ``_REASON_RULES`` (each rule a condition and the messages it adds);
* ``_clock_row``: per requested fixed clock pair, the observed and verified
  peaks, the verified geometries, the minimum-energy group per objective and
  the resource plateau;
* ``_recommendation``: per objective, the winner under the full-sweep
  throughput bar, the limits on its qualification, its input-size or resource
  plateau and its comparisons with the matched anchors;
* ``_selection_diagnostic``, ``_input_scaling``, ``_profiler_evidence``,
  ``_representative_trace``.

Keys, strings and their order are the reference's: evaluation.json and
evaluation.csv carry them.
"""
from __future__ import annotations

import hashlib
import json
import math
import re
from collections import Counter, defaultdict
from dataclasses import asdict, dataclass
from typing import Any, Callable, Mapping

from .contracts import SFU_CONTRACT_FIELDS
from .selections import (MEMORY, NONLINEAR, SFU, TENSOR, bar_metadata, coalescing_eligible, meets_bar,
                         peak_population_eligible, role_eligible)

OBJECTIVES = ("total", "operational_idle_increment", "paired_active_reference")
CANDIDATE_PLATEAUS = ("observed_plateau", "observed_problem_size_plateau", "observed_input_size_plateau")


def _num(value) -> float | None:
    if type(value) is float:                 # the common case: float() of an exact float is the float itself
        return value if value - value == 0.0 else None
    ok = isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value)
    return float(value) if ok else None


def canonical(value) -> str:
    """The compact sorted JSON that names strata and curves (its sha256 prefix is their id)."""
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False)


def _short_id(text: str) -> str:
    return hashlib.sha256(text.encode()).hexdigest()[:12]


# Rate and energy fields, units and scales per workload family.
_UNITS = {
    "sfu": {"rate": "throughput_sfu_instructions_s", "rate_unit": "G scalar SFU instructions/s", "rate_scale": 1e9,
            "energy_suffix": "pj_per_instruction", "energy_unit": "pJ/scalar SFU instruction"},
    "nonlinear": {"rate": "throughput_elements_s", "rate_unit": "Gelement/s", "rate_scale": 1e9,
                  "energy_suffix": "pj_per_element", "energy_unit": "pJ/element"},
    "tensor": {"rate": "throughput_ops_s", "rate_unit": "TFLOP/s", "rate_scale": 1e12,
               "energy_suffix": "pj_per_flop", "energy_unit": "pJ/FLOP"},
    "bytes": {"rate": "throughput_bytes_s", "rate_unit": "logical GB/s", "rate_scale": 1e9,
              "energy_suffix": "pj_per_logical_bit", "energy_unit": "pJ/logical bit"},
}


def units(workload) -> dict[str, Any]:
    family = ("sfu" if workload in SFU else "nonlinear" if workload in NONLINEAR else "tensor" if workload in TENSOR
              else "bytes")
    return dict(_UNITS[family])


@dataclass(frozen=True)
class EvaluationPolicy:
    """Gates of a candidate: plateau tolerance, resource levels, interval width (evaluation.py:118-130)."""
    plateau_tolerance_fraction: float = 0.05
    minimum_resource_levels: int = 3
    maximum_relative_ci_width: float = 0.10

    def __post_init__(self):
        if type(self.minimum_resource_levels) is not int or self.minimum_resource_levels < 3:
            raise ValueError("minimum_resource_levels must be an integer >=3")
        if not all(_num(v) is not None and 0 < v < 1
                   for v in (self.plateau_tolerance_fraction, self.maximum_relative_ci_width)):
            raise ValueError("Evaluation fractions must be finite and in (0,1)")


def component_stratum(group: Mapping) -> dict[str, Any]:
    keys = ("gpu_uuid", "workload", "benchmark_sha256", "measurement_stratum", "treatment_design_stratum",
            "experiment_contract")
    return {**{k: group.get(k) for k in keys}, "experiment_role": group.get("experiment_role", "legacy_unspecified")}


def _interval(group: Mapping, field: str):
    ci = (group.get("ci95") or {}).get(field)
    return ci if isinstance(ci, list) and len(ci) == 2 else None


def relative_width(group: Mapping, field: str) -> float | None:
    """Interval width over |median|; None when either is missing, the median is 0 or the ends are reversed."""
    value, ci = _num(group.get(field)), _interval(group, field)
    if value is None or value == 0 or ci is None or _num(ci[0]) is None or _num(ci[1]) is None or ci[0] > ci[1]:
        return None
    return (ci[1] - ci[0]) / abs(value)


def _precise(group: Mapping, field: str, policy: EvaluationPolicy) -> bool:
    width = relative_width(group, field)
    return width is not None and width <= policy.maximum_relative_ci_width


def capacity(group: Mapping) -> float | None:
    """The issue-resource level of a group: m n k for a GEMM, blocks x threads (x accumulators for Tensor)."""
    geometry = group.get("resource_geometry") or {}
    if group["workload"] == "gemm":
        dims = [_num(geometry.get(k)) for k in ("gemm_m", "gemm_n", "gemm_k")]
        return math.prod(dims) if all(d is not None and d > 0 for d in dims) else None
    blocks, threads = _num(geometry.get("blocks")), _num(geometry.get("threads"))
    if blocks is None or threads is None or blocks <= 0 or threads <= 0:
        return None
    if group["workload"] != "tensor":
        return blocks * threads
    return blocks * threads * (_num(geometry.get("tensor_accumulators")) or 1)


def _sfu_interval_positive(group: Mapping, metric: str) -> bool:
    ci = _interval(group, metric)
    return ci is not None and (_num(ci[0]) or 0) > 0


def qualified(group: Mapping, metric: str, rate: str, minimum_repeats: int, policy: EvaluationPolicy,
              require_hbm_candidate: bool = True) -> bool:
    """The numeric gates of a candidate: role, coalescing, SFU sign, HBM bandwidth, repeats,
    verification, a non-negative energy and precise energy and rate intervals."""
    if group.get("workload") in SFU and not (
            metric == "paired_active_reference_pj_per_instruction"
            and group.get("sfu_reference_delta_positive_optimum_eligible") is True
            and _sfu_interval_positive(group, metric)):
        return False
    if require_hbm_candidate and group.get("workload") == "hbm" and (group.get("hbm_bandwidth") or {}).get("eligible") is not True:
        return False
    energy = _num(group.get(metric))
    return (role_eligible(group) and coalescing_eligible(group)
            and group.get("valid_repeats", 0) >= minimum_repeats and group.get("verified_selection_eligible") is True
            and energy is not None and group[metric] >= 0
            and _precise(group, metric, policy) and _precise(group, rate, policy))


# ---------------------------------------------------------------------------- reasons
@dataclass
class _Ask:
    """One question: can ``group`` be a candidate for ``objective`` (energy ``metric``, ``rate``)?"""
    group: Mapping
    objective: str
    metric: str
    rate: str
    minimum_repeats: int
    policy: EvaluationPolicy

    @property
    def sfu(self) -> bool:
        return self.group.get("workload") in SFU


def _hbm_unqualified(a: _Ask) -> bool:
    return a.group.get("workload") == "hbm" and (a.group.get("hbm_bandwidth") or {}).get("eligible") is not True


def _hbm_messages(a: _Ask) -> list[str]:
    evidence = a.group.get("hbm_bandwidth") or {}
    return ["HBM clock-specific theoretical bandwidth threshold is unqualified",
            *evidence.get("reasons", ["missing_hbm_bandwidth_evidence"])]


def _energy(a: _Ask) -> float | None:
    return _num(a.group.get(a.metric))


def _fixed(message: str) -> Callable[[_Ask], list[str]]:
    return lambda a: [message]


# (condition, messages) in the order a point lists them.
_REASON_RULES: tuple[tuple[Callable[[_Ask], bool], Callable[[_Ask], list[str]]], ...] = (
    (lambda a: not role_eligible(a.group), _fixed("Diagnostic experiment role is excluded from energy characterization")),
    (_hbm_unqualified, _hbm_messages),
    (lambda a: not coalescing_eligible(a.group),
     lambda a: ["Coalesced memory-read energy evidence is unqualified",
                *(a.group.get("memory_coalescing") or {}).get("reasons", [])]),
    (lambda a: a.group.get("valid_repeats", 0) < a.minimum_repeats, _fixed("Insufficient valid repeats")),
    (lambda a: a.group.get("target_verified") is not True,
     lambda a: ["Target evidence: " + a.group.get("ncu_status", "unprofiled")]),
    (lambda a: a.group.get("count_energy_time_alignment_exact") is not True,
     _fixed("Work and energy windows are not exactly aligned")),
    (lambda a: not a.group.get("clock_comparison_controlled"),
     _fixed("Incoming clock policy is outside fixed-clock selection")),
    (lambda a: (_num(a.group.get(a.rate)) or 0) <= 0, _fixed("Positive sustained throughput is unavailable")),
    (lambda a: not _precise(a.group, a.rate, a.policy), _fixed("Throughput repeat uncertainty is unavailable or too wide")),
    (lambda a: not _precise(a.group, a.metric, a.policy), _fixed("Energy repeat uncertainty is unavailable or too wide")),
    (lambda a: _energy(a) is None, _fixed("Energy value is unavailable")),
    (lambda a: _energy(a) is not None and a.group[a.metric] < 0, _fixed("Negative operational contrast is diagnostic only")),
    (lambda a: a.objective != "total" and a.group.get(a.objective + "_eligible") is not True,
     _fixed("Matched baseline or balanced paired reference is unqualified")),
    (lambda a: a.sfu and a.objective != "paired_active_reference",
     _fixed("Board total and idle increment are diagnostics; direct SFU results use the paired register-loop contrast")),
    (lambda a: (a.sfu and a.objective == "paired_active_reference"
                and a.group.get("sfu_reference_delta_positive_optimum_eligible") is not True),
     _fixed("SFU contrast needs a qualified matched reference and a repeat interval strictly above zero to qualify as an energy candidate")),
    (lambda a: (a.sfu and a.objective == "paired_active_reference"
                and a.group.get("sfu_reference_delta_positive_optimum_eligible") is True
                and not _sfu_interval_positive(a.group, a.metric)),
     _fixed("A signed contrast whose interval reaches zero is diagnostic only")),
)


def eligibility_reasons(group: Mapping, objective: str, metric: str, rate: str, minimum_repeats: int,
                        policy: EvaluationPolicy) -> list[str]:
    ask = _Ask(group, objective, metric, rate, minimum_repeats, policy)
    return [message for condition, messages in _REASON_RULES if condition(ask) for message in messages(ask)]


# ---------------------------------------------------------------------------- plateaus and input-size curves
def _rate_population(groups, rate: str, minimum_repeats: int) -> list:
    """Groups whose valid rate may set a component's observed peak."""
    return [g for g in groups if peak_population_eligible(g) and g.get("valid_repeats", 0) >= minimum_repeats
            and (_num(g.get(rate)) or 0) > 0]


def _stable(rates: list, peak, fraction: float, policy: EvaluationPolicy) -> bool:
    return (peak is not None and min(rates) >= fraction * peak
            and (max(rates) - min(rates)) / max(rates) <= policy.plateau_tolerance_fraction)


def resource_plateau(groups: list, rate: str, fraction: float, minimum_repeats: int, policy: EvaluationPolicy) -> dict:
    """Do the highest tested issue-resource levels (verified, precise) reach similar rates near the peak?"""
    observed = _rate_population(groups, rate, minimum_repeats)
    peak = max((g[rate] for g in observed), default=None)
    best_at: dict = {}
    for g in observed:
        level = capacity(g)
        if level is None or g.get("verified_selection_eligible") is not True or not _precise(g, rate, policy):
            continue
        if level not in best_at or best_at[level][rate] < g[rate]:
            best_at[level] = g
    top = sorted(best_at)[-policy.minimum_resource_levels:]
    chosen = [best_at[level] for level in top]
    rates = [g[rate] for g in chosen]
    stable = len(rates) >= policy.minimum_resource_levels and _stable(rates, peak, fraction, policy)
    gemm = bool(groups) and groups[0]["workload"] == "gemm"
    return {"status": ("observed_problem_size_plateau" if gemm else "observed_plateau") if stable else "inconclusive",
            "reason": "highest tested issue-resource levels have similar verified throughput" if stable else
                      "three verified, precise increasing resource levels near the complete observed peak are required",
            "resource_axis": "GEMM m × n × k; problem-size evidence, vendor algorithms can change" if gemm else
                             "blocks × threads × accumulators (Tensor); blocks × threads otherwise",
            "resource_levels": top, "group_ids": [g["group_id"] for g in chosen], "throughputs": rates,
            "observed_peak": peak, "hardware_saturation_proven": False}


def _input_contract(group: Mapping) -> Mapping:
    return group.get("sfu_contract" if group.get("workload") in SFU else "nonlinear_contract") or {}


def input_q(group: Mapping):
    """The input size Q: active register lanes (SFU) or input elements (complete functions)."""
    return _input_contract(group).get("sfu_lanes" if group.get("workload") in SFU else "input_elements")


def launch_record(group: Mapping) -> dict[str, Any]:
    contract, geometry = _input_contract(group), group.get("resource_geometry") or {}
    sfu = ({"sfu_lanes": contract.get("sfu_lanes"), "sfu_chains": contract.get("sfu_chains"),
            "q_scope": "active scalar register lanes, not function output elements"}
           if group.get("workload") in SFU else {})
    return {"input_elements": input_q(group), **sfu, "grid_mode": contract.get("grid_mode"),
            "blocks": geometry.get("blocks"), "threads": geometry.get("threads"),
            "block_completion_count_source": contract.get("block_completion_count_source")}


_Q_VARYING = {"input_elements", "sfu_lanes", "working_set_bytes", "blocks"}


def input_curve_signature(group: Mapping) -> str | None:
    """What an input-size curve holds fixed (everything but Q and what Q sets); None for a group on
    no curve (not an auto-grid complete function or SFU loop, uncontrolled clocks, a non-integral Q)."""
    sfu, contract = group.get("workload") in SFU, _input_contract(group)
    on_curve = (role_eligible(group) and group.get("workload") in NONLINEAR | SFU and contract.get("grid_mode") == "auto"
                and contract.get("math_implementation") == ("ptx_approx_register_v1" if sfu else "cuda_fp32_q_grid_v2")
                and group.get("clock_comparison_controlled"))
    q = _num(input_q(group)) if on_curve else None
    if q is None or q <= 0 or q != int(q):
        return None
    fixed = lambda d, drop: {k: v for k, v in (d or {}).items() if k not in drop}  # noqa: E731
    stratum = component_stratum(group)
    stratum["experiment_contract"] = fixed(group.get("experiment_contract"), _Q_VARYING)
    return canonical({**stratum, ("sfu_contract" if sfu else "nonlinear_contract"): fixed(contract, _Q_VARYING),
                      "config": fixed(group.get("config"), _Q_VARYING | {"clock_selection_policy", "clock_selection_reasons"}),
                      "resource_geometry": fixed(group.get("resource_geometry"), {"blocks"})})


def _accepted(g: Mapping, objective: str, metric: str, rate: str, minimum_repeats: int, policy: EvaluationPolicy) -> bool:
    return (qualified(g, metric, rate, minimum_repeats, policy)
            and not eligibility_reasons(g, objective, metric, rate, minimum_repeats, policy))


def input_size_plateau(candidate: Mapping, peers: list, objective: str, metric: str, rate: str, fraction: float,
                       minimum_repeats: int, policy: EvaluationPolicy) -> dict:
    """Does the winner's Q sit among the largest tested Q levels of its curve, each with a
    qualified near-peak rate?  Unqualified valid rates still count toward the peak and the Q
    levels, so dropping a failed high-Q point cannot make a lower plateau."""
    observed = _rate_population(peers, rate, minimum_repeats)
    peak = max((g[rate] for g in observed), default=None)
    top = sorted({input_q(g) for g in observed})[-policy.minimum_resource_levels:]
    chosen = []
    for q in top:
        level = [g for g in observed if input_q(g) == q and _accepted(g, objective, metric, rate, minimum_repeats, policy)]
        if level:
            chosen.append(max(level, key=lambda g: (g[rate], g["group_id"])))
    rates = [g[rate] for g in chosen]
    q_selected = input_q(candidate)
    spread = (max(rates) - min(rates)) / max(rates) if rates else None
    stable = (len(top) >= policy.minimum_resource_levels and len(chosen) == len(top) and q_selected in top
              and _stable(rates, peak, fraction, policy))
    sfu = candidate.get("workload") in SFU
    return {"status": "observed_input_size_plateau" if stable else "inconclusive",
            "curve_id": _short_id(input_curve_signature(candidate)),
            "reason": "The selected Q lies in the largest tested Q levels with precise, verified near-peak throughput" if stable else
                      f"The selected Q must belong to the {policy.minimum_resource_levels} largest observed Q levels, each qualified and stable near the complete matching-curve peak",
            "resource_axis": "active register lanes Q at fixed threads, chains, clocks, iterations and SFU primitive" if sfu else
                             "input elements Q at fixed threads, clocks, iterations and function definition",
            "input_elements_levels": top, "selected_input_elements": q_selected,
            **({"sfu_lanes_levels": top, "selected_sfu_lanes": q_selected} if sfu else {}),
            "group_ids": [g["group_id"] for g in chosen], "throughputs": rates,
            "observed_peak": peak, "relative_throughput_spread": spread,
            "hardware_saturation_proven": False,
            "scope": "Observed input-size stability only; Q-dependent energy values remain separate and SFU or GPU saturation is not established"}


def objective_measured(group: Mapping, objective: str) -> bool:
    """A valid observation of the objective, whether or not it can win."""
    if objective == "total":
        return group.get("valid_repeats", 0) > 0
    if objective == "paired_active_reference" and group.get("workload") in SFU:
        return group.get("sfu_reference_delta_measurement_valid") is True
    return group.get(objective + "_eligible") is True


def _by_objective(fn: Callable[[str], Any]) -> dict[str, Any]:
    return {o: fn(o) for o in OBJECTIVES}


# ---------------------------------------------------------------------------- plan coverage
_TRIAL_ID = re.compile(r"[A-Za-z0-9][A-Za-z0-9._-]{0,199}")


def check_trial_ids(trials: list) -> None:
    """Unique, filename-safe trial ids (runner.py:30-40): the ValueError the runner raises."""
    seen: set = set()
    for index, trial in enumerate(trials):
        identifier = trial.get("trial_id") if isinstance(trial, dict) else None
        if not isinstance(identifier, str) or not _TRIAL_ID.fullmatch(identifier):
            raise ValueError(f"Unsafe or missing trial_id at record {index}: {identifier!r}")
        if identifier in seen:
            raise ValueError(f"Duplicate trial_id: {identifier}")
        seen.add(identifier)


def _bound_to_plan(trial: Mapping, row: Mapping, workload: str, plan: Mapping) -> bool:
    """Does the analysed trial carry the planned row's identity, clocks, parameters and arm order?"""
    device = plan.get("device") or {}
    config, clocks = trial.get("config", {}), row.get("clocks", {})
    order = (row.get("treatment_protocol") or {}).get("order")
    checks = (
        trial.get("workload") == workload,
        device.get("uuid") is None or trial.get("gpu_uuid") == device.get("uuid"),
        trial.get("experiment_role", "legacy_unspecified") == row.get("experiment_role", "legacy_unspecified"),
        trial.get("repeat_index") == row.get("repeat"),
        device.get("benchmark_sha256") is None or trial.get("benchmark_sha256") == device.get("benchmark_sha256"),
        trial.get("condition_id") == row.get("condition_id"),
        config.get("graphics_clock_mhz") == clocks.get("graphics_mhz") and config.get("memory_clock_mhz") == clocks.get("memory_mhz"),
        all(config.get(k) == v for k, v in row.get("parameters", {}).items()),
        order is None or (trial.get("paired_active_reference_protocol") or {}).get("order") == order,
    )
    return all(checks)


def plan_coverage(summary: Mapping, plan, plan_validator: Callable[[Mapping], None] | None = None) -> dict:
    """Which planned trials the summary holds, per workload, bound by identity and conditions.

    ``plan_validator`` is the planner's execution policy check (runner.validate_plan_execution,
    whose clock-grid rules belong to the planner); its ValueError text becomes
    ``plan_policy_error``.  Without one, no policy error is reported."""
    if plan is None:
        return {"status": "unknown", "reason": "No plan supplied; measured data alone cannot establish sweep completeness",
                "by_workload": {}}
    if not isinstance(plan, dict) or not isinstance(plan.get("trials"), list):
        raise ValueError("Evaluation plan must be an object with a trials list")
    check_trial_ids(plan["trials"])
    policy_error = None
    if plan_validator is not None:
        try:
            plan_validator(plan)
        except ValueError as exc:
            policy_error = str(exc)
    actual = {t["trial_id"]: t for t in summary["trials"] if t.get("trial_id") is not None}
    planned = plan.get("trials", [])
    by_workload: dict[str, dict] = {}
    mismatched_all: list = []
    for workload in sorted({t["workload"] for t in planned}):
        rows = [t for t in planned if t["workload"] == workload]
        missing = [r["trial_id"] for r in rows if r["trial_id"] not in actual]
        present = [(r, actual[r["trial_id"]]) for r in rows if r["trial_id"] in actual]
        mismatched = [r["trial_id"] for r, t in present if not _bound_to_plan(t, r, workload, plan)]
        invalid = [r["trial_id"] for r, t in present if not t.get("valid")]
        mismatched_all += mismatched
        by_workload[workload] = {"planned_trials": len(rows), "observed_trials": len(rows) - len(missing),
                                 "missing_trial_ids": missing, "invalid_trial_ids": invalid,
                                 "mismatched_trial_ids": mismatched,
                                 "status": "incomplete" if missing or mismatched else
                                           "complete_with_rejections" if invalid else "complete"}
    unexpected = sorted(set(actual) - {t["trial_id"] for t in planned})
    duplicates = summary.get("duplicate_trial_ids_ignored", [])
    incomplete = (policy_error or unexpected or mismatched_all or duplicates
                  or any(w["missing_trial_ids"] for w in by_workload.values()))
    return {"status": "incomplete" if incomplete else "complete",
            "plan_policy_error": policy_error, "study_design": plan.get("study_design", "legacy_unspecified"),
            "clock_policy": plan.get("clock_sweep_coverage"), "by_workload": by_workload,
            "unexpected_trial_ids": unexpected, "duplicate_trial_ids": duplicates,
            "note": "Coverage binds trial IDs, GPU, workload, clocks, parameters and paired-arm order; target evidence is assessed separately"}


# ---------------------------------------------------------------------------- matched anchors
_NOT_GEOMETRY = {"graphics_clock_mhz", "memory_clock_mhz", "clock_selection_policy", "clock_selection_reasons",
                 "seconds", "warmup_seconds", "idle_seconds"}


def _match_signature(group: Mapping) -> str:
    config = {k: v for k, v in group["config"].items() if k not in _NOT_GEOMETRY}
    return canonical({"config": config, "resource_geometry": group.get("resource_geometry")})


def _is_anchor(group: Mapping, candidate: Mapping, anchor: str) -> bool:
    config = group["config"]
    if anchor == "factory_default":
        return "advertised_default_fixed_pair" in config.get("clock_selection_reasons", [])
    return config.get("graphics_clock_mhz") == 1110 and config.get("memory_clock_mhz") == candidate["config"].get("memory_clock_mhz")


def anchor_comparison(candidate: Mapping, groups: list, objective: str, rate: str, metric: str, minimum_repeats: int,
                      policy: EvaluationPolicy, anchor: str) -> dict:
    """The winner against the same geometry, input and seed at the anchor clocks (the advertised
    default pair, or exactly 1110 MHz at the winner's memory clock)."""
    signature = _match_signature(candidate)
    refs = [g for g in groups if _match_signature(g) == signature and _is_anchor(g, candidate, anchor)]
    if len(refs) != 1:
        return {"status": "inconclusive", "reason": "A unique matched geometry/input/seed reference is missing", "anchor": anchor}
    ref = refs[0]
    usable = ((objective == "total" or ref.get(objective + "_eligible") is True)
              and qualified(ref, metric, rate, minimum_repeats, policy, require_hbm_candidate=False) and ref[metric] > 0)
    if not usable:
        return {"status": "inconclusive", "reason": "Reference lacks qualified positive energy, repeats, exact counts or profile evidence",
                "anchor": anchor, "reference_group_id": ref["group_id"], "reference_hbm_bandwidth": ref.get("hbm_bandwidth")}
    same = candidate["group_id"] == ref["group_id"]
    c_lo, c_hi = candidate["ci95"][metric]
    r_lo, r_hi = ref["ci95"][metric]
    bounds = [1 - c_hi / r_lo, 1 - c_lo / r_hi] if r_lo > 0 else None
    evidence = ("same_condition" if same else "resolved_improvement" if bounds and bounds[0] > 0
                else "resolved_regression" if bounds and bounds[1] < 0 else "difference_unresolved")
    return {"status": "available", "anchor": anchor, "reference_group_id": ref["group_id"],
            "reference_hbm_bandwidth": ref.get("hbm_bandwidth"),
            "reference_bandwidth_scope": "A qualified measured anchor remains available for comparison even when it does not meet the HBM candidate bandwidth threshold" if ref.get("workload") == "hbm" else None,
            "energy_reduction_fraction": 0 if same else 1 - candidate[metric] / ref[metric],
            "throughput_ratio": 1 if same else candidate[rate] / ref[rate],
            "energy_reduction_interval_from_ci_endpoints": [0, 0] if same else bounds,
            "evidence": evidence,
            "uncertainty_note": "CI endpoint envelope is descriptive, not a calibrated ratio confidence interval; sensor systematic error is excluded"}


# ---------------------------------------------------------------------------- representative trace
_TRACE_FIELDS = ("t_s", "power_w", "graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz", "temperature_c")


def _thinned(n: int) -> list[int]:
    """At most 96 sample indices, evenly spread over n samples with both ends kept."""
    if n <= 1:
        return list(range(n))
    points = min(96, n)
    return sorted({round(i * (n - 1) / min(95, n - 1)) for i in range(points)})


def trace_points(record: Mapping) -> list | None:
    """A record's display trace: at most 96 samples per phase (None when its phases are not a dict)."""
    phases = record.get("phases") or {}
    if not isinstance(phases, dict):
        return None
    points = []
    for name, phase in phases.items():
        samples = phase.get("samples", [])
        points += [{"phase": name, **{k: _num(samples[i].get(k)) for k in _TRACE_FIELDS}}
                   for i in _thinned(len(samples)) if isinstance(samples[i], dict)]
    return points


def representative_trace(groups: list, analyzed: Mapping, traces: Mapping) -> dict | None:
    """The median-energy valid repeat of the best-repeated group with a trace (``traces``: trial id ->
    trace_points of its record, None or absent when it has none)."""
    for group in sorted(groups, key=lambda g: (-g.get("valid_repeats", 0), g["group_id"])):
        valid = sorted((analyzed[i] for i in group["trial_ids"] if i in analyzed and analyzed[i].get("valid")),
                       key=lambda t: t.get("total_energy_j") or 0)
        if not valid:
            continue
        trial = valid[len(valid) // 2]
        points = traces.get(trial["trial_id"])
        if points is None:
            continue
        return {"trial_id": trial["trial_id"], "group_id": group["group_id"], "points": points,
                "note": "One valid repeat; at most 96 observed samples per phase for display only. Energy uses original samples and exact complete epochs."}
    return None


class _LazyTraces(dict):
    """trial id -> trace_points of the last record with that id, computed on first use."""

    def __init__(self, records):
        super().__init__()
        self.records = {r.get("trial_id"): r for r in records}

    def get(self, trial_id, default=None):
        if trial_id not in self:
            record = self.records.get(trial_id)
            self[trial_id] = None if record is None else trace_points(record)
        return dict.get(self, trial_id, default)


# ---------------------------------------------------------------------------- one component
@dataclass
class _Context:
    policy: EvaluationPolicy
    minimum_repeats: int
    minimum_geometries: int
    fraction: float
    near_fraction: float
    plan: Any
    coverage: dict
    analyzed: dict
    traces: Mapping
    input_curves: dict


def _anchor_tags(group: Mapping, ctx: _Context) -> list[str]:
    config = group["config"]
    tags = list(config.get("clock_selection_reasons", []))
    if ctx.plan is not None:
        default = (ctx.plan.get("clock_sweep_coverage") or {}).get("advertised_default") or {}
        pair = (config.get("graphics_clock_mhz"), config.get("memory_clock_mhz"))
        if default.get("status") == "included" and pair == (default.get("graphics_mhz"), default.get("memory_mhz")):
            tags.append("advertised_default_fixed_pair")
    if config.get("graphics_clock_mhz") == 1110:
        tags.append("required_exact_1110_mhz")
    return sorted(set(tags))


def _sfu_delta(group: Mapping) -> dict:
    return {"measurement_valid": group.get("sfu_reference_delta_measurement_valid"),
            "positive_optimum_eligible": group.get("sfu_reference_delta_positive_optimum_eligible"),
            "ci_crosses_zero": group.get("sfu_reference_delta_ci_crosses_zero"),
            "signed_pj_per_instruction": group.get("sfu_reference_delta_pj_per_instruction"),
            "issues": group.get("sfu_reference_delta_issues"),
            "uncertainty": group.get("sfu_reference_delta_uncertainty"),
            "hardware_attribution_proven": False}


def _point(group: Mapping, config: Mapping, trials: list, u: dict, ctx: _Context) -> dict:
    """The component's row for one group: ``group`` carries its anchor tags in its config's
    clock_selection_reasons, ``config`` is the group's own config."""
    workload, rate, suffix = group["workload"], u["rate"], u["energy_suffix"]
    ci = group.get("ci95", {})
    geometry, coalescing = group.get("memory_access_geometry") or {}, group.get("memory_coalescing") or {}
    energy_field = lambda o: o + "_" + suffix  # noqa: E731
    return {
        "group_id": group["group_id"], "requested_graphics_mhz": config.get("graphics_clock_mhz"),
        "experiment_role": group.get("experiment_role", "legacy_unspecified"),
        "memory_access_geometry": group.get("memory_access_geometry"), "memory_coalescing": group.get("memory_coalescing"),
        "memory_stride_words": geometry.get("stride_words"), "memory_lane_stride_bytes": geometry.get("lane_stride_bytes"),
        "memory_observed_sector_efficiency_pct": coalescing.get("observed_sector_efficiency_pct"),
        "memory_coalescing_energy_eligible": group.get("memory_coalescing_energy_eligible"),
        "hbm_memory_power": group.get("hbm_memory_power"), "hbm_bandwidth": group.get("hbm_bandwidth"),
        **bar_metadata(group, ctx.fraction),
        "energy_peak_population_eligible": peak_population_eligible(group),
        "requested_memory_mhz": config.get("memory_clock_mhz"), "achieved_graphics_mhz": group.get("graphics_clock_mhz"),
        "achieved_sm_mhz": group.get("sm_clock_mhz"), "achieved_memory_mhz": group.get("memory_clock_mhz"),
        "resource_capacity": capacity(group), "geometry": group.get("resource_geometry"),
        "anchor_tags": list(group["config"]["clock_selection_reasons"]),
        "ncu_status": group.get("ncu_status"), "valid_repeats": group.get("valid_repeats", 0),
        "rejected_repeats": group["repeats"] - group["valid_repeats"],
        "quality_issues": dict(Counter(issue for t in trials for issue in t.get("issues", []))),
        "relative_ci_widths": {f: relative_width(group, f) for f in (rate, *map(energy_field, OBJECTIVES))},
        "rate": group.get(rate), "rate_ci95": ci.get(rate),
        "energies": _by_objective(lambda o: group.get(energy_field(o))),
        "energy_ci95": _by_objective(lambda o: ci.get(energy_field(o))),
        "objective_eligible": _by_objective(lambda o: o == "total" or group.get(o + "_eligible") is True),
        "objective_measurement_valid": _by_objective(lambda o: objective_measured(group, o)),
        "eligibility_reasons": _by_objective(
            lambda o: eligibility_reasons(group, o, energy_field(o), rate, ctx.minimum_repeats, ctx.policy)),
        "tensor_dense_peak_fraction": group.get("tensor_utilization_vs_dense_clock_peak"),
        "measurement_diagnostics": group.get("measurement_diagnostics"),
        "nonlinear_launch": launch_record(group) if workload in NONLINEAR else None,
        "sfu_launch": launch_record(group) if workload in SFU else None,
        "sfu_reference_delta": _sfu_delta(group) if workload in SFU else None,
        "sfu_reference_diagnostics": group.get("sfu_reference_delta_diagnostics"),
        "row_width": (group.get("nonlinear_contract") or {}).get("row_width"),
        "pj_per_row": _by_objective(lambda o: group.get(o + "_pj_per_row")),
        "config": config}


def _profiler_evidence(group: Mapping, trials: list) -> dict:
    checks: dict = {}
    for t in trials:
        for check in (t.get("ncu_assessment") or {}).get("checks", []):
            checks[(check.get("name"), check.get("status"))] = check
    return {"group_id": group["group_id"], "status": group.get("ncu_status"), "checks": list(checks.values()),
            "sampled_numerical_checks": [t["numerical_validation"] for t in trials if t.get("numerical_validation")],
            "traffic_amplification": [t["ncu_assessment"]["traffic_amplification"] for t in trials
                                      if (t.get("ncu_assessment") or {}).get("traffic_amplification")],
            "profile_rates": [t["profile_rates_summary"] for t in trials if t.get("profile_rates_summary")]}


def _latency_points(group: Mapping, trials: list) -> list:
    config = group["config"]
    return [{"trial_id": t["trial_id"], "group_id": group["group_id"], "sm_id": sm,
             "offset_bytes": config.get("offset_bytes", 0), "graphics_mhz": config.get("graphics_clock_mhz"),
             "memory_mhz": config.get("memory_clock_mhz"), "cycles_per_access": probe["cycles_per_access"]}
            for t in trials for sm, probe in (t.get("latency_probe") or {}).get("per_sm", {}).items()
            if t.get("valid") and (_num(probe.get("cycles_per_access")) or 0) > 0]


def _winner(groups: list, metric: str, rate: str):
    return min(groups, key=lambda g: (g[metric], -g[rate], g["group_id"]), default=None)


def _clock_row(pair: tuple, rows: list, u: dict, ctx: _Context, candidates: dict) -> dict:
    """One requested clock pair: peaks, verified geometries, per-objective minimum, plateau;
    the objective candidates found here are added to ``candidates``."""
    rate = u["rate"]
    observed = _rate_population(rows, rate, ctx.minimum_repeats)
    peak = max((g[rate] for g in observed), default=None)
    verified = [g for g in observed if g.get("verified_selection_eligible")]
    geometries = len({canonical(g["resource_geometry"]) for g in verified})
    minimum = {}
    for objective in OBJECTIVES:
        metric = objective + "_" + u["energy_suffix"]
        eligible = [g for g in verified if geometries >= ctx.minimum_geometries
                    and qualified(g, metric, rate, ctx.minimum_repeats, ctx.policy)
                    and meets_bar(g, rate, peak, ctx.fraction)
                    and (objective == "total" or g.get(objective + "_eligible") is True)]
        best = _winner(eligible, metric, rate)
        minimum[objective] = best["group_id"] if best else None
        candidates[objective].extend(eligible)
    if all(input_curve_signature(g) is not None for g in rows):
        plateau = {"status": "not_applicable_q_grid",
                   "reason": "Q determines the grid; selected-candidate evidence uses a matched input-size curve",
                   "hardware_saturation_proven": False}
    else:
        plateau = resource_plateau(rows, rate, ctx.fraction, ctx.minimum_repeats, ctx.policy)
    return {"graphics_mhz": pair[0], "memory_mhz": pair[1], "observed_peak": peak,
            "verified_peak": max((g[rate] for g in verified), default=None), "verified_geometry_count": geometries,
            "minimum_energy_group_ids": minimum, "plateau": plateau, "plateau_is_candidate_gate": rows[0]["workload"] != "hbm"}


def _qualification_limits(winner: Mapping, workload: str, plateau: Mapping, on_curve: bool, ctx: _Context) -> list[str]:
    """Why a winner is only a provisional candidate (none: a qualified observed candidate)."""
    coverage = ctx.coverage
    of_workload = coverage.get("by_workload", {}).get(workload, {})
    limits = (
        (coverage["status"] != "complete" or of_workload.get("status") not in ("complete", "complete_with_rejections"),
         "planned coverage is incomplete or unknown"),
        (coverage.get("study_design") != "energy_sweep", "a complete energy-sweep plan is required"),
        (workload in SFU and _input_contract(winner).get("grid_mode") != "auto",
         "a Q-derived automatic grid is required; fixed-grid SFU results remain diagnostic or provisional"),
        (workload != "hbm" and plateau["status"] not in CANDIDATE_PLATEAUS,
         "input-size plateau is inconclusive" if on_curve else "resource plateau is inconclusive"),
    )
    return [text for failed, text in limits if failed]


_DIAGNOSTIC_ROLE = ("Explicit diagnostic experiments are excluded from energy characterization and its observed peak")
_SFU_BOARD = ("Board total and idle increment are not direct SFU energy results; the primary estimator is the signed "
              "matched register-loop contrast")


def _recommendation(objective: str, groups: list, u: dict, candidates: dict, clocks: list, observed_peak,
                    tagged: list, ctx: _Context) -> dict:
    workload, rate = groups[0]["workload"], u["rate"]
    metric = objective + "_" + u["energy_suffix"]
    if not role_eligible(groups[0]):
        return {"objective": objective, "status": "diagnostic_only", "group_id": None, "reason": _DIAGNOSTIC_ROLE}
    if workload in SFU and objective != "paired_active_reference":
        return {"objective": objective, "status": "diagnostic_only", "group_id": None, "reason": _SFU_BOARD}
    eligible = [g for g in candidates[objective] if meets_bar(g, rate, observed_peak, ctx.fraction)]
    if not eligible:
        gate = ("the HBM clock-specific theoretical bandwidth threshold" if workload == "hbm"
                else "the full observed throughput threshold")
        return {"objective": objective, "status": "no_qualified_candidate", "group_id": None,
                "reason": "No candidate meets profile/count/repeat/CI/geometry gates and " + gate}
    winner = _winner(eligible, metric, rate)
    pair = (winner["config"]["graphics_clock_mhz"], winner["config"]["memory_clock_mhz"])
    clock = next(c for c in clocks if (c["graphics_mhz"], c["memory_mhz"]) == pair)
    curve = input_curve_signature(winner)
    plateau = (input_size_plateau(winner, ctx.input_curves[curve], objective, metric, rate, ctx.fraction,
                                  ctx.minimum_repeats, ctx.policy) if curve is not None else clock["plateau"])
    limits = _qualification_limits(winner, workload, plateau, curve is not None, ctx)
    saturation = ({"status": "clock_specific_theoretical_bandwidth_threshold_met", "hardware_saturation_proven": False,
                   "hbm_bandwidth": winner.get("hbm_bandwidth"), "resource_plateau_diagnostic": plateau}
                  if workload == "hbm" else plateau)
    compare = lambda anchor: anchor_comparison(winner, tagged, objective, rate, metric, ctx.minimum_repeats,  # noqa: E731
                                               ctx.policy, anchor)
    return {"objective": objective, "group_id": winner["group_id"],
            "status": "provisional_candidate" if limits else "qualified_observed_candidate",
            "qualification_limits": limits, "saturation_evidence": saturation, **bar_metadata(winner, ctx.fraction),
            "energy": winner[metric], "energy_ci95": winner["ci95"].get(metric),
            "throughput_fraction_of_observed_peak": winner[rate] / observed_peak,
            "near_optimum_group_ids": [g["group_id"] for g in eligible if g[metric] <= winner[metric] * (1 + ctx.near_fraction)],
            "factory_default_comparison": compare("factory_default"), "exact_1110_comparison": compare("exact_1110")}


def _selection_diagnostic(objective: str, workload: str, u: dict, candidates: dict, recommendation: Mapping,
                          observed_peak, ctx: _Context) -> dict:
    """The lowest own-clock candidate against the winner under the full-sweep throughput bar."""
    metric, rate = objective + "_" + u["energy_suffix"], u["rate"]
    own = _winner(candidates[objective], metric, rate)
    energy = recommendation.get("energy")
    hbm = workload == "hbm"
    if hbm:
        reason = "HBM candidates use the clock-specific theoretical bandwidth threshold; observed-peak ratios do not exclude candidates"
    elif own is None:
        reason = "No qualified own-clock candidate"
    elif observed_peak and own[rate] < ctx.fraction * observed_peak:
        reason = "The lowest own-clock candidate falls below the full-sweep throughput threshold"
    else:
        reason = "The lowest own-clock candidate meets the full-sweep throughput threshold"
    return {"objective": objective,
            "lowest_own_clock_candidate_group_id": own["group_id"] if own else None,
            "lowest_own_clock_candidate_energy": own[metric] if own else None,
            "own_clock_candidate_global_throughput_fraction": own[rate] / observed_peak if own and observed_peak else None,
            "global_constraint_candidate_group_id": recommendation.get("group_id"),
            "global_constraint_candidate_energy": energy,
            "global_constraint_energy_over_own_clock_energy": energy / own[metric] if own and own[metric] > 0 and energy is not None else None,
            "reason": reason,
            "scope": "HBM absolute bandwidth admission; observed-peak ratios and resource plateau are diagnostics only" if hbm else
                     "Same count/profile/repeat/CI/geometry gates and own-clock throughput bar; comparing the added full-sweep throughput constraint, not correcting energy or proving saturation"}


def _input_scaling(groups: list, u: dict, ctx: _Context) -> dict:
    """Every input-size curve the component's groups lie on, one row per Q point."""
    rate, suffix = u["rate"], u["energy_suffix"]
    curves = []
    for signature in sorted({s for g in groups if (s := input_curve_signature(g)) is not None}):
        rows = []
        for g in sorted(ctx.input_curves[signature], key=lambda g: (input_q(g), g["group_id"])):
            ci = g.get("ci95", {})
            reasons = _by_objective(lambda o: eligibility_reasons(g, o, o + "_" + suffix, rate, ctx.minimum_repeats, ctx.policy))
            rows.append({"group_id": g["group_id"], **launch_record(g),
                         "requested_graphics_mhz": g["config"].get("graphics_clock_mhz"),
                         "requested_memory_mhz": g["config"].get("memory_clock_mhz"),
                         "rate": g.get(rate), "rate_ci95": ci.get(rate),
                         "energies": _by_objective(lambda o: g.get(o + "_" + suffix)),
                         "objective_measurement_valid": _by_objective(lambda o: objective_measured(g, o)),
                         "energy_ci95": _by_objective(lambda o: ci.get(o + "_" + suffix)),
                         "valid_repeats": g.get("valid_repeats", 0), "ncu_status": g.get("ncu_status"),
                         "eligible": _by_objective(lambda o: not reasons[o] and qualified(
                             g, o + "_" + suffix, rate, ctx.minimum_repeats, ctx.policy)),
                         "eligibility_reasons": reasons})
        curves.append({"curve_id": _short_id(signature), "signature": json.loads(signature), "rows": rows})
    return {"curves": curves,
            "scope": "Each curve holds GPU, binary, measurement/input definition, requested fixed clocks, threads, chains and iterations constant; only Q changes. Q is active register lanes for direct SFU and input elements for complete functions. Energies and recommendations remain separate per Q. Stable throughput is not proof of hardware saturation."}


def _correctness_scope(workload: str) -> str:
    if workload in SFU:
        return "native scalar SFU instruction retention and target-path evidence; register-loop contrast is not isolated physical SFU rail energy"
    if workload in NONLINEAR:
        return "distributed CPU-double output samples before/after measurement; not exhaustive"
    if workload in TENSOR:
        return "finite output samples and issued-operation accounting; full mathematical reference not established"
    return "issued addresses/counts and path evidence; no physical partition identity or exhaustive bytewise output proof"


def _interpretation(workload: str) -> str:
    if workload == "l2_latency":
        return "dependent-load latency map; no near/far or energy optimum"
    if workload == "control":
        return "active issue-control reference; no component energy optimum"
    if workload in SFU:
        return "signed treatment/control contrast per scalar SFU instruction; negative or zero-crossing contrasts remain diagnostics, and board total/idle are separate diagnostics"
    return "measured whole-device energy of the stated implementation; component rail energy is not isolated"


def _component(key: str, groups: list, ctx: _Context) -> dict:
    stratum = json.loads(key)
    workload = stratum["workload"]
    u = units(workload)
    rate = u["rate"]
    points, evidence, latency = [], [], []
    by_clock: dict = defaultdict(list)
    for group in groups:
        trials = [ctx.analyzed[i] for i in group["trial_ids"] if i in ctx.analyzed]
        config = group["config"]
        # The anchor tags ride in a copy's config, for the matched comparisons.
        tagged = {**group, "config": {**config, "clock_selection_reasons": _anchor_tags(group, ctx)}}
        points.append(_point(tagged, config, trials, u, ctx))
        if tagged.get("clock_comparison_controlled"):
            by_clock[(config.get("graphics_clock_mhz"), config.get("memory_clock_mhz"))].append(tagged)
        evidence.append(_profiler_evidence(tagged, trials))
        latency += _latency_points(tagged, trials)
    candidates: dict = defaultdict(list)
    clocks = [_clock_row(pair, rows, u, ctx, candidates) for pair, rows in sorted(by_clock.items())]
    observed_peak = max((c["observed_peak"] for c in clocks if c["observed_peak"] is not None), default=None)
    for point in points:
        pair = (point["requested_graphics_mhz"], point["requested_memory_mhz"])
        clock = next((c for c in clocks if (c["graphics_mhz"], c["memory_mhz"]) == pair), None)
        extra = []
        if clock and clock["verified_geometry_count"] < ctx.minimum_geometries:
            extra.append("Too few verified execution geometries at this clock")
        if workload != "hbm" and observed_peak and point["rate"] is not None and point["rate"] < ctx.fraction * observed_peak:
            extra.append("Below the all-valid observed throughput threshold")
        for reasons in point["eligibility_reasons"].values():
            reasons.extend(extra)
    tagged_all = [g for rows in by_clock.values() for g in rows]
    recommendations = [_recommendation(o, groups, u, candidates, clocks, observed_peak, tagged_all, ctx) for o in OBJECTIVES]
    diagnostics = [_selection_diagnostic(o, workload, u, candidates, r, observed_peak, ctx)
                   for o, r in zip(OBJECTIVES, recommendations)]
    sfu = workload in SFU
    counts = Counter("valid" if ctx.analyzed[i].get("valid") else "invalid"
                     for g in groups for i in g["trial_ids"] if i in ctx.analyzed)
    return {"component_id": _short_id(key), "stratum": stratum, "gpu_name": groups[0].get("gpu_name"), "units": u,
            "primary_objective": "paired_active_reference" if sfu else "total",
            "primary_estimator": "(treatment mean power - matched register-loop control mean power) / treatment scalar SFU instruction rate" if sfu else None,
            "trial_counts": dict(counts), "points": points, "clocks": clocks, "observed_peak": observed_peak,
            "recommendations": recommendations, "energy_selection_diagnostics": diagnostics,
            "input_scaling": _input_scaling(groups, u, ctx),
            "profiler_evidence": evidence, "latency_points": latency,
            "correctness_scope": _correctness_scope(workload),
            "measurement_example": representative_trace(groups, ctx.analyzed, ctx.traces),
            "interpretation": _interpretation(workload)}


LIMITS = (
    "All optima are restricted to observed supported clocks and tested configurations.",
    "Bootstrap intervals measure repeat variation, not sensor calibration accuracy.",
    "Profiler counter rates use replay busy time and are never energy-run sustained throughput.",
    "HBM candidates use sustained logical payload versus clock-specific DDR theory from complete measured memory-clock and CUDA bus-width evidence; this is not simultaneous physical DRAM utilization. Observed-peak ratios and resource plateaus are HBM diagnostics only.",
    "Compare the same energy objective and denominator. Total/idle ratios and replay traffic amplification diagnose differences; they do not rescale the measured energy.",
    "Diagnostic experiments and known noncoalesced memory reads cannot define energy optima or their peak. Unknown counter proof for a structurally coalesced run does not lower the observed throughput bar.",
    "A resource plateau is empirical evidence; it does not prove hardware saturation or pure component energy.",
    "Nonlinear auto-grid candidates use matching Q-scaling evidence; input-size stability does not prove SFU or GPU saturation, and energy is never pooled across Q.",
    "Direct SFU results use a signed matched register-loop power contrast per scalar instruction. Different execution durations or register use limit physical attribution; total and idle estimates are board diagnostics.",
    "Factory default means the advertised fixed clock pair; incoming driver policy is a separate reference.",
)


def evaluate(summary: Mapping, plan=None, policy=None, raw_records=(), plan_validator=None,
             traces: Mapping | None = None) -> dict[str, Any]:
    """The evaluation of a summary (evaluation.py:436): components, plan coverage, limits.

    ``raw_records`` are the runner's records (for the representative traces), or ``traces`` their
    trace_points by trial id (what a sharded caller gathers instead of whole records);
    ``plan_validator`` is the planner's execution policy check (see plan_coverage)."""
    policy = policy if isinstance(policy, EvaluationPolicy) else EvaluationPolicy(**(policy or {}))
    selection = summary["selection_policy"]
    coverage = plan_coverage(summary, plan, plan_validator)
    strata: dict = defaultdict(list)
    curves: dict = defaultdict(list)
    for group in summary.get("groups", []):
        strata[canonical(component_stratum(group))].append(group)
        signature = input_curve_signature(group)
        if signature is not None:
            curves[signature].append(group)
    ctx = _Context(policy=policy, minimum_repeats=selection["min_repeats"], minimum_geometries=selection["min_geometries"],
                   fraction=selection["throughput_fraction"], near_fraction=selection.get("near_optimum_fraction", 0.05),
                   plan=plan, coverage=coverage, analyzed={t["trial_id"]: t for t in summary["trials"]},
                   traces=traces if traces is not None else _LazyTraces(raw_records), input_curves=curves)
    components = [_component(key, groups, ctx) for key, groups in sorted(strata.items())]
    return {"schema_version": 1,
            "policy": {**asdict(policy), "throughput_fraction": ctx.fraction,
                       "hbm_bandwidth_fraction": selection.get("hbm_bandwidth_fraction", 0.80),
                       "minimum_repeats": ctx.minimum_repeats, "minimum_geometries": ctx.minimum_geometries},
            "coverage": coverage, "components": components,
            "missing_workloads": sorted(set(coverage.get("by_workload", {})) - {c["stratum"]["workload"] for c in components}),
            "limits": list(LIMITS)}


# ---------------------------------------------------------------------------- files
EVALUATION_CSV_FIELDS = (
    "component_id", "gpu_uuid", "workload", "contract", "group_id", "objective", "requested_graphics_mhz",
    "requested_memory_mhz", "achieved_sm_mhz", "geometry", "anchor_tags", "ncu_status", "valid_repeats",
    "rejected_repeats", "throughput", "rate_unit", "energy", "energy_unit", "energy_ci95", "objective_eligible",
    "objective_measurement_valid", "recommendation_status", "quality_issues", "eligibility_reasons",
    "dense_tensor_peak_fraction", "row_width", "pj_per_row", "measurement_diagnostics", "nonlinear_launch", "sfu_launch",
    "sfu_reference_delta", "sfu_reference_diagnostics", "experiment_role", "memory_stride_words",
    "memory_lane_stride_bytes", "memory_observed_sector_efficiency_pct", "memory_coalescing_energy_eligible",
    "energy_peak_population_eligible", "memory_access_geometry", "memory_coalescing", "hbm_memory_power", "hbm_bandwidth",
    "hbm_bandwidth_status", "hbm_logical_gbps", "hbm_theoretical_gbps", "hbm_fraction_of_theoretical",
    "hbm_minimum_fraction", "hbm_bandwidth_reasons", "hbm_bandwidth_warnings", "hbm_physical_dram_utilization_measured")

HBM_POWER_CSV_FIELDS = (
    "component_id", "group_id", "gpu_uuid", "gpu_name", "requested_graphics_mhz", "requested_memory_mhz", "geometry",
    "experiment_contract", "ncu_status", "status", "scope", "source", "semantics", "measurement_valid",
    "normalization_valid", "incremental_valid", "observed_repeats", "valid_repeats", "normalized_repeats",
    "incremental_repeats", "power_w", "energy_j", "idle_power_w", "incremental_power_w", "incremental_energy_j",
    "pj_per_logical_bit", "incremental_pj_per_logical_bit", "ci95", "freshness_status", "freshness_verified",
    "maximum_sensor_age_s", "freshness_maximum_age_s", "board_invalid_repeats", "duplicate_repeats_excluded",
    "board_power_w", "board_total_pj_per_logical_bit", "issues", "incremental_issues")


def _cell(value):
    return json.dumps(value, ensure_ascii=False) if isinstance(value, (list, dict)) else value


def _scaled(value, scale):
    return value / scale if value is not None else None


def evaluation_rows(evaluation: Mapping):
    """evaluation.csv: one row per (component point, objective)."""
    for c in evaluation["components"]:
        status_of = {(r.get("group_id"), r["objective"]): r["status"] for r in c["recommendations"]}
        stratum, u = c["stratum"], c["units"]
        for p in c["points"]:
            bandwidth = p.get("hbm_bandwidth") or {}
            for o, energy in p["energies"].items():
                yield {**{k: p.get(k) for k in EVALUATION_CSV_FIELDS},
                       "component_id": c["component_id"], "gpu_uuid": stratum["gpu_uuid"], "workload": stratum["workload"],
                       "contract": stratum["experiment_contract"], "objective": o,
                       "throughput": _scaled(p["rate"], u["rate_scale"]), "rate_unit": u["rate_unit"],
                       "energy": energy, "energy_unit": u["energy_unit"], "energy_ci95": p["energy_ci95"][o],
                       "objective_eligible": p["objective_eligible"][o],
                       "objective_measurement_valid": p["objective_measurement_valid"][o],
                       "eligibility_reasons": p.get("eligibility_reasons", {}).get(o, []),
                       "dense_tensor_peak_fraction": p.get("tensor_dense_peak_fraction"),
                       "pj_per_row": p.get("pj_per_row", {}).get(o),
                       "recommendation_status": status_of.get((p["group_id"], o)),
                       "hbm_bandwidth_status": bandwidth.get("status"),
                       "hbm_logical_gbps": _scaled(bandwidth.get("sustained_logical_bytes_s"), 1e9),
                       "hbm_theoretical_gbps": _scaled(bandwidth.get("theoretical_bytes_s"), 1e9),
                       "hbm_fraction_of_theoretical": bandwidth.get("fraction_of_theoretical"),
                       "hbm_minimum_fraction": bandwidth.get("minimum_fraction"),
                       "hbm_bandwidth_reasons": bandwidth.get("reasons"),
                       "hbm_bandwidth_warnings": bandwidth.get("warnings", []),
                       "hbm_physical_dram_utilization_measured": bandwidth.get("physical_dram_utilization_measured")}


def hbm_power_rows(evaluation: Mapping):
    """hbm-memory-power.csv: one row per HBM point, its memory-rail analysis beside the board's."""
    for c in evaluation["components"]:
        if c["stratum"]["workload"] != "hbm":
            continue
        for p in c["points"]:
            sensor = p.get("hbm_memory_power") or {"status": "unavailable", "scope": "memory",
                                                   "issues": ["missing_sensor_analysis"]}
            board = (p.get("measurement_diagnostics") or {}).get("power_contributions") or {}
            yield {**{k: sensor.get(k) for k in HBM_POWER_CSV_FIELDS},
                   **{k: p.get(k) for k in ("group_id", "requested_graphics_mhz", "requested_memory_mhz", "geometry", "ncu_status")},
                   "component_id": c["component_id"], "gpu_uuid": c["stratum"]["gpu_uuid"], "gpu_name": c.get("gpu_name"),
                   "experiment_contract": c["stratum"].get("experiment_contract"),
                   "board_power_w": board.get("total_w"), "board_total_pj_per_logical_bit": p["energies"].get("total")}


def _write_csv(path, fields, rows) -> None:
    import csv
    with path.open("w", newline="") as stream:
        writer = csv.DictWriter(stream, fieldnames=list(fields))
        writer.writeheader()
        for row in rows:
            writer.writerow({k: _cell(v) for k, v in row.items()})


def write_evaluation(evaluation: Mapping, output) -> dict[str, str]:
    """evaluation.json and evaluation.csv (and hbm-memory-power.csv when an HBM component exists),
    as the reference's dashboard.write_evaluation writes them; its HTML view is not produced."""
    from pathlib import Path
    out = Path(output)
    out.mkdir(parents=True, exist_ok=True)
    paths = {"evaluation_json": out / "evaluation.json", "evaluation_csv": out / "evaluation.csv"}
    paths["evaluation_json"].write_text(json.dumps(evaluation, indent=2, ensure_ascii=False, allow_nan=False) + "\n")
    _write_csv(paths["evaluation_csv"], EVALUATION_CSV_FIELDS, evaluation_rows(evaluation))
    if any(c["stratum"]["workload"] == "hbm" for c in evaluation["components"]):
        paths["hbm_memory_power_csv"] = out / "hbm-memory-power.csv"
        _write_csv(paths["hbm_memory_power_csv"], HBM_POWER_CSV_FIELDS, hbm_power_rows(evaluation))
    return {k: str(v) for k, v in paths.items()}
