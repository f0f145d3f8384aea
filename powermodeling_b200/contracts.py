"""Count contracts that a workload record must satisfy to be analysed.

A powerbench ``result`` (or ``active_reference_result``) record states its
launch geometry and the work it counted, in total and per measure epoch.
Each contract here is data: which identity fields a record family must carry
(``Expect``), which execution parameters must lie in range (bounds tables) and
which counted quantities must equal products of the geometry (``Relation``),
in the record and in every epoch.  One evaluator (``_Audit``) reads the
counts and turns every unmet expectation into the issue string analysis
output carries; the strings and the rules they name are the reference's
(sfu.py:23-115, memory.py:114-144, nonlinear.py:22-128), pinned by fixtures
the reference's own count_issues produced (tests/golden/count_contracts.json.gz,
tests/golden/nonlinear_contract.json.gz).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Mapping

SFU_WORKLOADS = {"sfu_ex2", "sfu_lg2", "sfu_rcp", "sfu_rsqrt", "sfu_sqrt", "sfu_tanh"}
SFU_REFERENCE_KIND = "register_loop_without_sfu"
SFU_CONTRACT_FIELDS = ("sfu_lanes", "sfu_chains", "sfu_primitive", "sfu_input_policy",
                       "iterations_per_launch", "grid_mode", "math_implementation",
                       "kernel_implementation_version", "block_completion_count_source", "sfu_ptx_opcode",
                       "sfu_approximate", "sfu_flush_to_zero", "sfu_exponent_base")
NONLINEAR_WORKLOADS = {"exp", "tanh", "silu", "rmsnorm", "softmax"}
NONLINEAR_ROW_WORKLOADS = {"rmsnorm", "softmax"}

# Record families by kernel_implementation_version: memory reads count one
# access per thread-iteration, the four-stream write/copy kernel four.
MEMORY_FAMILIES = {
    "scalar_single_stream_read_v3": (1, ("read",)),
    "scalar_single_stream_read_v2": (1, ("read",)),
    "scalar_four_stream_write_copy_v1": (4, ("write", "copy")),
}


def _number(value) -> float | None:
    """A finite int or float (bools excluded) as a float."""
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
        return None
    return float(value)


def _whole(value) -> bool:
    """A non-negative integral count (int or float, bools excluded)."""
    return (not isinstance(value, bool) and isinstance(value, (int, float)) and math.isfinite(value)
            and value >= 0 and value == int(value))


def _product(*factors):
    """Product of the factors, None when any is unknown."""
    out = 1
    for f in factors:
        if f is None:
            return None
        out *= f
    return out


def _same(value, expected) -> bool:
    """Equality for an identity field; True, False and None compare by identity."""
    return value is expected if expected is None or isinstance(expected, bool) else value == expected


@dataclass(frozen=True)
class Expect:
    """Identity fields a record family must carry; one issue for any mismatch."""
    issue: str
    fields: tuple            # (field, expected value) pairs


@dataclass(frozen=True)
class Relation:
    """counted field == product of named quantities (or a constant), per scope."""
    name: str
    field: str
    expected: tuple | int    # quantity names, or a constant


class _Audit:
    """Reads a record's counts and collects the issues its contract raises.

    invalid: prefix of the issue for a count that is not a non-negative
    integer; disagree: prefix of the issue for a relation that does not hold
    (relative 1e-9, absolute 1e-6)."""

    def __init__(self, invalid: str, disagree: str):
        self.invalid, self.disagree = invalid, disagree
        self.issues: list[str] = []

    def raise_if(self, condition, issue: str) -> None:
        if condition:
            self.issues.append(issue)

    def count(self, obj: Mapping, key: str):
        value = obj.get(key)
        if _whole(value):
            return value
        self.issues.append(self.invalid + key)
        return None

    def agree(self, name: str, actual, expected) -> None:
        if actual is None or expected is None or not math.isclose(actual, expected, rel_tol=1e-9, abs_tol=1e-6):
            self.issues.append(self.disagree + name)

    def expect(self, obj: Mapping, expectations, prefix: str = "") -> None:
        for e in expectations:
            if any(not _same(obj.get(f), v) for f, v in e.fields):
                self.issues.append(prefix + e.issue)

    def relations(self, obj: Mapping, relations, quantities: Mapping, label: str) -> None:
        for r in relations:
            expected = r.expected if isinstance(r.expected, int) else _product(*(quantities[q] for q in r.expected))
            self.agree(label + r.name, self.count(obj, r.field), expected)

    def result(self) -> list[str]:
        return sorted(set(self.issues))


def _epochs(record: Mapping):
    """The record's measure epochs when they are a non-empty list, else None."""
    epochs = record.get("measure_epochs")
    return epochs if isinstance(epochs, list) and epochs else None


def _checked_values_missing(record: Mapping) -> bool:
    checked = (record.get("numerical_validation") or {}).get("checked_values")
    return _number(checked) is None or checked <= 0


# ---------------------------------------------------------------------------- SFU
_SFU_PTX = {"ex2": "ex2.approx.ftz.f32", "lg2": "lg2.approx.ftz.f32", "rcp": "rcp.approx.ftz.f32",
            "rsqrt": "rsqrt.approx.ftz.f32", "sqrt": "sqrt.approx.ftz.f32", "tanh": "tanh.approx.f32"}
_SFU_SLOTS = ("launches", "lanes", "iterations", "chains")
# Execution parameters and the range each must lie in.
_SFU_BOUNDS = (("lanes", lambda v: bool(v)), ("chains", lambda v: v in (1, 4, 8)),
               ("iterations", lambda v: bool(v) and v <= 2 ** 32), ("blocks", lambda v: bool(v) and v <= 1_000_000),
               ("launches", lambda v: bool(v)), ("threads", lambda v: v is not None and 32 <= v <= 1024 and not v % 32))


def _sfu_identity(primitive: str, reference: bool) -> tuple:
    return (
        Expect("unsupported_implementation",
               (("kernel_implementation_version", "sfu_register_control_v1" if reference else "sfu_register_recurrence_v1"),)),
        Expect("unsupported_math_contract", () if reference else (("math_implementation", "ptx_approx_register_v1"),)),
        Expect("unsupported_primitive_or_input_policy",
               (("sfu_input_policy", "feedback_xor_iteration_mantissa_0p5_1_v1"), ("sfu_primitive", primitive))),
        Expect("unsupported_ptx_definition",
               (("sfu_ptx_opcode", _SFU_PTX[primitive]), ("sfu_approximate", True), ("sfu_flush_to_zero", primitive != "tanh"),
                ("sfu_exponent_base", 2 if primitive in ("ex2", "lg2") else None))),
        Expect("unsupported_count_source", (("block_completion_count_source", "synchronized_completed_launches"),)),
        Expect("unsupported_reference_definition",
               (("workload", "control"), ("reference_kind", SFU_REFERENCE_KIND)) if reference else ()),
    )


def _sfu_relations(reference: bool) -> tuple:
    """What a treatment launch counts (one MUFU op per lane, iteration and chain) and what its
    paired register-loop reference counts (loop slots, no SFU work)."""
    work = 0 if reference else _SFU_SLOTS
    return ((Relation("completed_ctas", "admitted_blocks", ("launches", "blocks")),
             Relation("instructions", "sfu_instructions", work), Relation("operations", "operations", work))
            + ((Relation("reference_loop_slots", "reference_loop_slots", _SFU_SLOTS),) if reference else ())
            + (Relation("logical_bytes", "logical_bytes", 0), Relation("elements", "elements", 0)))


def sfu_count_issues(benchmark: Mapping, workload: str, *, reference: bool = False) -> list[str]:
    """Issues of an SFU treatment record, or (reference=True) of its paired active-reference record."""
    if workload not in SFU_WORKLOADS:
        return []
    prefix = "sfu_reference_" if reference else "sfu_"
    audit = _Audit(prefix + "invalid_count:", prefix + "count_disagreement:")
    audit.expect(benchmark, _sfu_identity(workload[len("sfu_"):], reference), prefix)
    geometry = {name: audit.count(benchmark, key) for name, key in (
        ("lanes", "sfu_lanes"), ("chains", "sfu_chains"), ("iterations", "iterations_per_launch"),
        ("blocks", "blocks"), ("threads", "threads"), ("launches", "kernel_launches"))}
    audit.raise_if(not all(ok(geometry[name]) for name, ok in _SFU_BOUNDS), prefix + "invalid_execution_parameters")
    mode = benchmark.get("grid_mode")
    audit.raise_if(mode not in ("auto", "fixed"), prefix + "invalid_grid_mode")
    if mode == "auto" and geometry["lanes"] and geometry["threads"]:
        audit.agree("auto_grid_blocks", geometry["blocks"], math.ceil(geometry["lanes"] / geometry["threads"]))
    if "batch_launches" in benchmark:
        geometry["batch_launches"] = audit.count(benchmark, "batch_launches")
        audit.raise_if(not geometry["batch_launches"] or geometry["batch_launches"] > 65536, prefix + "invalid_batch_launches")
    else:
        geometry["batch_launches"] = None
    relations = _sfu_relations(reference)

    def scope(obj: Mapping, label: str) -> None:
        quantities = dict(geometry, launches=audit.count(obj, "kernel_launches"))
        audit.relations(obj, relations, quantities, label)
        if "batches" in obj:
            audit.agree(label + "batch_kernel_launches", quantities["launches"],
                        _product(audit.count(obj, "batches"), geometry["batch_launches"]))

    scope(benchmark, "total_")
    epochs = _epochs(benchmark)
    if epochs is None:
        audit.issues.append(prefix + "missing_measure_epochs")
    else:
        for epoch in epochs:
            if not isinstance(epoch, dict):
                audit.issues.append(prefix + "invalid_epoch")
                continue
            for name in SFU_CONTRACT_FIELDS + ("batch_launches",):
                audit.raise_if(name in epoch and epoch[name] != benchmark.get(name),
                               prefix + "epoch_contract_disagreement:" + name)
            scope(epoch, "epoch_")
            audit.raise_if(epoch.get("counts_exact") is not True, prefix + "inexact_epoch")
        summed = ("kernel_launches", "sfu_instructions", "operations") + (("reference_loop_slots",) if reference else ())
        for name in summed:
            parts = [audit.count(epoch, name) for epoch in epochs if isinstance(epoch, dict)]
            audit.agree("epoch_total_" + name, None if None in parts else sum(parts), audit.count(benchmark, name))
    sanity = benchmark.get("sanity") or {}
    audit.raise_if(sanity.get("finite_output_sample") is False, prefix + "output_sanity_failed")
    if not reference:
        audit.raise_if(sanity.get("numerical_validation_passed") is not True, "sfu_numerical_validation_failed_or_missing")
        audit.raise_if(_checked_values_missing(benchmark), "sfu_missing_one_step_reference_checks")
    return audit.result()


# ---------------------------------------------------------------------------- memory
def memory_count_issues(benchmark: Mapping, workload: str) -> list[str]:
    """Issues of a scalar memory record: its operations and logical bytes against admitted blocks x
    threads x iterations x accesses per thread-iteration (x 4 bytes, x 2 for a copy), in total
    and per epoch, in that order."""
    family = MEMORY_FAMILIES.get(benchmark.get("kernel_implementation_version"))
    if workload not in ("l1", "l2", "hbm") or family is None:
        return []
    accesses, access_values = family
    access = benchmark.get("access")
    issues = []
    if access not in access_values:
        issues.append("memory_contract_access_implementation_mismatch")
    if _number(benchmark.get("memory_accesses_per_thread_iteration")) != accesses:
        issues.append("memory_contract_accesses_per_iteration_mismatch")
    per_block = [_number(benchmark.get(k)) for k in ("threads", "iterations_per_launch")]
    if any(v is None or v <= 0 or not v.is_integer() for v in per_block):
        issues.append("memory_contract_invalid_execution_parameters")
        return issues
    bytes_per_access = 8 if access == "copy" else 4
    scopes = [("total", benchmark)]
    epochs = benchmark.get("measure_epochs", benchmark.get("work_epochs"))
    if isinstance(epochs, list):
        scopes += [(f"epoch_{i}", e) for i, e in enumerate(epochs) if isinstance(e, dict)]
    for label, obj in scopes:
        admitted = _number(obj.get("admitted_blocks"))
        if admitted is None or admitted < 0 or not admitted.is_integer():
            issues.append("memory_contract_missing_or_invalid_admissions:" + label)
            continue
        operations = admitted * per_block[0] * per_block[1] * accesses
        for field, expected in (("operations", operations), ("logical_bytes", operations * bytes_per_access)):
            actual = _number(obj.get(field))
            if actual is None or actual < 0 or abs(actual - expected) > max(1.0, abs(expected) * 1e-6):
                issues.append(f"memory_contract_count_disagreement:{label}:{field}")
    return issues


# ---------------------------------------------------------------------------- nonlinear
def nonlinear_bytes_per_element(workload) -> int:
    """Logical bytes of one output element: RMSNorm reads x twice, gamma once and writes y;
    softmax reads x three times and writes y (nonlinear.py:17-19)."""
    return 16 if workload in NONLINEAR_ROW_WORKLOADS else 8


_Q_GRID = {"math_implementation": "cuda_fp32_q_grid_v2", "kernel_implementation_version": "fp32_complete_nonlinear_q_grid_v2"}
_NONLINEAR_MATH = {"cuda_fp32_standard_streaming_v1", "cuda_fp32_q_grid_v2"}


def _row_quotient(elements, width, row):
    """Row evaluations an element count implies: elements / width for row functions, else 0."""
    if not row:
        return 0
    return elements / width if elements is not None and width else None


def nonlinear_count_issues(benchmark: Mapping, workload: str) -> list[str]:
    """Denominator checks of a complete-nonlinear-function record.

    An element is one output value (a whole row reduction included for RMSNorm
    and softmax).  Q-grid records must account for every completed launch:
    launches x Q x iterations elements, launches x blocks CTAs, per epoch and
    in total; records of the first streaming implementation are checked per
    admitted block."""
    if workload not in NONLINEAR_WORKLOADS:
        return []
    row = workload in NONLINEAR_ROW_WORKLOADS
    per_element = nonlinear_bytes_per_element(workload)
    audit = _Audit("invalid_nonlinear_count:", "nonlinear_count_disagreement:")
    elements = audit.count(benchmark, "elements")
    audit.raise_if(elements is not None and elements <= 0, "missing_nonlinear_elements")
    audit.agree("operations_are_elements", audit.count(benchmark, "operations"), elements)
    audit.agree("logical_bytes", audit.count(benchmark, "logical_bytes"), _product(elements, per_element))
    width = audit.count(benchmark, "row_width")
    if row:
        audit.raise_if(width is None or not 1 <= width <= 65536 or width != int(width), "invalid_nonlinear_row_width")
    else:
        audit.agree("row_width", width, 0)
    audit.agree("row_evaluations", audit.count(benchmark, "row_evaluations"), _row_quotient(elements, width, row))
    g = {k: audit.count(benchmark, key) for k, key in (("blocks", "blocks"), ("ws", "working_set_bytes"),
                                                       ("iterations", "iterations_per_launch"), ("admitted", "admitted_blocks"))}
    q_grid = any(benchmark.get(f) == v for f, v in _Q_GRID.items())
    g.update(q=None, launches=None, batch_launches=None)
    if q_grid:
        audit.raise_if(any(benchmark.get(f) != v for f, v in _Q_GRID.items()), "unsupported_nonlinear_q_grid_implementation")
        audit.raise_if(benchmark.get("block_completion_count_source") != "synchronized_completed_launches",
                       "unsupported_nonlinear_block_completion_count_source")
        g["q"], threads, g["launches"] = (audit.count(benchmark, k) for k in ("input_elements", "threads", "kernel_launches"))
        if "batch_launches" in benchmark:
            g["batch_launches"] = audit.count(benchmark, "batch_launches")
            audit.raise_if(not g["batch_launches"], "invalid_nonlinear_batch_launches")
        if "batches" in benchmark:
            audit.agree("completed_batch_kernel_launches", g["launches"],
                        _product(audit.count(benchmark, "batches"), g["batch_launches"]))
        ws, q = g["ws"], g["q"]
        audit.raise_if(ws is None or ws <= 0 or ws % 4, "invalid_nonlinear_input_word_alignment")
        audit.agree("input_elements", q, None if ws is None else ws / 4)
        audit.raise_if(q is None or q <= 0 or (width and row and q % width), "incomplete_nonlinear_input_or_row")
        audit.raise_if(threads is None or not 32 <= threads <= 1024 or threads % 32, "invalid_nonlinear_threads")
        mode = benchmark.get("grid_mode")
        audit.raise_if(mode not in ("auto", "fixed"), "invalid_nonlinear_grid_mode")
        if mode == "auto" and q and threads and (not row or width):
            audit.agree("auto_grid_blocks", g["blocks"], q / width if row else math.ceil(q / threads))
        audit.raise_if(not g["blocks"] or g["blocks"] > 1_000_000 or not g["iterations"] or not g["launches"],
                       "missing_nonlinear_execution_counts")
        if g["launches"] is not None and g["blocks"] is not None:
            audit.agree("completed_launch_admissions", g["admitted"], g["launches"] * g["blocks"])
        audit.agree("completed_launch_elements", elements, _product(g["launches"], q, g["iterations"]))
    elif g["blocks"] and g["ws"] and g["iterations"] and g["admitted"]:
        # the first streaming implementation: contiguous per-CTA slices of the input
        audit.agree("admission_elements", elements, g["admitted"] * (g["ws"] / 4 / g["blocks"]) * g["iterations"])
        audit.raise_if(g["ws"] % (4 * g["blocks"] * (width if row and width else 1)), "incomplete_nonlinear_block_slice_or_row")
    else:
        audit.issues.append("missing_nonlinear_execution_counts")
    audit.raise_if(benchmark.get("math_implementation") not in _NONLINEAR_MATH or benchmark.get("input_precision") != "fp32",
                   "unsupported_nonlinear_math_contract")
    audit.raise_if(workload == "rmsnorm" and (benchmark.get("rms_epsilon") != 1e-5 or benchmark.get("affine_gamma") is not True),
                   "unsupported_rmsnorm_definition")
    audit.raise_if((benchmark.get("sanity") or {}).get("numerical_validation_passed") is not True,
                   "nonlinear_numerical_validation_failed_or_missing")
    audit.raise_if(_checked_values_missing(benchmark), "missing_nonlinear_numerical_reference_checks")
    epochs = _epochs(benchmark)
    if epochs is None:
        audit.issues.append("missing_nonlinear_measure_epochs")
        return audit.result()
    for epoch in epochs:
        if not isinstance(epoch, dict):
            audit.issues.append("invalid_nonlinear_epoch")
            continue
        e = audit.count(epoch, "elements")
        audit.agree("epoch_operations_are_elements", audit.count(epoch, "operations"), e)
        audit.agree("epoch_logical_bytes", audit.count(epoch, "logical_bytes"), _product(e, per_element))
        audit.agree("epoch_rows", audit.count(epoch, "row_evaluations"), e / width if e is not None and width and row else 0)
        if q_grid:
            launches = audit.count(epoch, "kernel_launches")
            if "batches" in epoch:
                audit.agree("epoch_completed_batch_kernel_launches", launches,
                            _product(audit.count(epoch, "batches"), g["batch_launches"]))
            audit.agree("epoch_completed_launch_admissions", audit.count(epoch, "admitted_blocks"), _product(launches, g["blocks"]))
            audit.agree("epoch_completed_launch_elements", e, _product(launches, g["q"], g["iterations"]))
        audit.raise_if(epoch.get("counts_exact") is not True, "inexact_nonlinear_measure_epoch")

    def total(key: str):
        """Sum of an epoch field over the epochs that carry a number in it."""
        return sum(ep.get(key, 0) for ep in epochs if isinstance(ep, dict) and isinstance(ep.get(key), (int, float)))

    audit.agree("epoch_total_elements", total("elements"), elements)
    if q_grid:
        audit.agree("epoch_total_kernel_launches", total("kernel_launches"), g["launches"])
    return audit.result()


def contract_fields(benchmark: Mapping, workload: str) -> dict[str, Any] | None:
    """The SFU contract fields of a record, as the analysis reports them (None for other workloads)."""
    return {f: benchmark.get(f) for f in SFU_CONTRACT_FIELDS} if workload in SFU_WORKLOADS else None


__all__ = ["SFU_WORKLOADS", "SFU_REFERENCE_KIND", "SFU_CONTRACT_FIELDS", "NONLINEAR_WORKLOADS", "MEMORY_FAMILIES",
           "sfu_count_issues", "memory_count_issues", "nonlinear_count_issues", "nonlinear_bytes_per_element",
           "contract_fields", "Expect", "Relation"]
