"""Count contracts that a workload record must satisfy to be analysed.

Restates the reference's powermodeling/sfu.py:count_issues (sfu.py:23-115),
powermodeling/memory.py:count_issues (memory.py:114-144) and
powermodeling/nonlinear.py:count_issues (nonlinear.py:22-128): the issues a
powerbench ``result`` (or ``active_reference_result``) record raises when its
reported counts disagree with its own launch geometry.  libpmb200's workload
front end emits records that pass these checks; analyze_trial applies them.
The issue strings are the reference's, since analysis output carries them.
"""
from __future__ import annotations

import math

SFU_WORKLOADS = {"sfu_ex2", "sfu_lg2", "sfu_rcp", "sfu_rsqrt", "sfu_sqrt", "sfu_tanh"}
SFU_KERNEL_IMPLEMENTATION = "sfu_register_recurrence_v1"
SFU_CONTROL_IMPLEMENTATION = "sfu_register_control_v1"
SFU_MATH_IMPLEMENTATION = "ptx_approx_register_v1"
SFU_INPUT_POLICY = "feedback_xor_iteration_mantissa_0p5_1_v1"
SFU_REFERENCE_KIND = "register_loop_without_sfu"
SFU_COUNT_SOURCE = "synchronized_completed_launches"
SFU_PTX_OPCODES = {p: p + ".approx.ftz.f32" for p in ("ex2", "lg2", "rcp", "rsqrt", "sqrt")}
SFU_PTX_OPCODES["tanh"] = "tanh.approx.f32"
SFU_CONTRACT_FIELDS = ("sfu_lanes", "sfu_chains", "sfu_primitive", "sfu_input_policy",
                       "iterations_per_launch", "grid_mode", "math_implementation",
                       "kernel_implementation_version", "block_completion_count_source", "sfu_ptx_opcode",
                       "sfu_approximate", "sfu_flush_to_zero", "sfu_exponent_base")

MEMORY_SINGLE_STREAM_READ_VERSIONS = {"scalar_single_stream_read_v3", "scalar_single_stream_read_v2"}
MEMORY_FOUR_STREAM_WRITE_COPY = "scalar_four_stream_write_copy_v1"
MEMORY_VERSIONS = MEMORY_SINGLE_STREAM_READ_VERSIONS | {MEMORY_FOUR_STREAM_WRITE_COPY}
NONLINEAR_WORKLOADS = {"exp", "tanh", "silu", "rmsnorm", "softmax"}


def _number(value):
    return float(value) if isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value) else None


def sfu_count_issues(benchmark, workload, *, reference=False) -> list[str]:
    if workload not in SFU_WORKLOADS:
        return []
    issues: list[str] = []
    prefix = "sfu_reference_" if reference else "sfu_"

    def integral(key, obj=benchmark):
        value = obj.get(key)
        if (isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value)
                or value < 0 or value != int(value)):
            issues.append(prefix + "invalid_count:" + key)
            return None
        return value

    def agree(name, actual, expected):
        if actual is None or expected is None or not math.isclose(actual, expected, rel_tol=1e-9, abs_tol=1e-6):
            issues.append(prefix + "count_disagreement:" + name)

    primitive = workload.removeprefix("sfu_")
    if benchmark.get("kernel_implementation_version") != (SFU_CONTROL_IMPLEMENTATION if reference else SFU_KERNEL_IMPLEMENTATION):
        issues.append(prefix + "unsupported_implementation")
    if not reference and benchmark.get("math_implementation") != SFU_MATH_IMPLEMENTATION:
        issues.append(prefix + "unsupported_math_contract")
    if benchmark.get("sfu_input_policy") != SFU_INPUT_POLICY or benchmark.get("sfu_primitive") != primitive:
        issues.append(prefix + "unsupported_primitive_or_input_policy")
    if (benchmark.get("sfu_ptx_opcode") != SFU_PTX_OPCODES[primitive]
            or benchmark.get("sfu_approximate") is not True
            or benchmark.get("sfu_flush_to_zero") is not (primitive != "tanh")
            or benchmark.get("sfu_exponent_base") != (2 if primitive in ("ex2", "lg2") else None)):
        issues.append(prefix + "unsupported_ptx_definition")
    if benchmark.get("block_completion_count_source") != SFU_COUNT_SOURCE:
        issues.append(prefix + "unsupported_count_source")
    if reference and (benchmark.get("workload") != "control" or benchmark.get("reference_kind") != SFU_REFERENCE_KIND):
        issues.append(prefix + "unsupported_reference_definition")
    lanes, chains, iterations, blocks, threads, launches = (integral(k) for k in (
        "sfu_lanes", "sfu_chains", "iterations_per_launch", "blocks", "threads", "kernel_launches"))
    if (not lanes or chains not in (1, 4, 8) or not iterations or iterations > 2 ** 32
            or not blocks or blocks > 1000000 or not launches
            or threads is None or not 32 <= threads <= 1024 or threads % 32):
        issues.append(prefix + "invalid_execution_parameters")
    mode = benchmark.get("grid_mode")
    if mode not in ("auto", "fixed"):
        issues.append(prefix + "invalid_grid_mode")
    elif mode == "auto" and lanes and threads:
        agree("auto_grid_blocks", blocks, math.ceil(lanes / threads))
    batch_launches = integral("batch_launches") if "batch_launches" in benchmark else None
    if "batch_launches" in benchmark and (not batch_launches or batch_launches > 65536):
        issues.append(prefix + "invalid_batch_launches")

    def counts(obj, label):
        count = integral("kernel_launches", obj)
        slots = count * lanes * iterations * chains if None not in (count, lanes, iterations, chains) else None
        agree(label + "completed_ctas", integral("admitted_blocks", obj),
              count * blocks if count is not None and blocks is not None else None)
        agree(label + "instructions", integral("sfu_instructions", obj), 0 if reference else slots)
        agree(label + "operations", integral("operations", obj), 0 if reference else slots)
        if reference:
            agree(label + "reference_loop_slots", integral("reference_loop_slots", obj), slots)
        agree(label + "logical_bytes", integral("logical_bytes", obj), 0)
        agree(label + "elements", integral("elements", obj), 0)
        if "batches" in obj:
            batches = integral("batches", obj)
            agree(label + "batch_kernel_launches", count,
                  batches * batch_launches if batches is not None and batch_launches is not None else None)

    counts(benchmark, "total_")
    epochs = benchmark.get("measure_epochs")
    if not isinstance(epochs, list) or not epochs:
        issues.append(prefix + "missing_measure_epochs")
    else:
        for epoch in epochs:
            if not isinstance(epoch, dict):
                issues.append(prefix + "invalid_epoch")
                continue
            for name in SFU_CONTRACT_FIELDS + ("batch_launches",):
                if name in epoch and epoch[name] != benchmark.get(name):
                    issues.append(prefix + "epoch_contract_disagreement:" + name)
            counts(epoch, "epoch_")
            if epoch.get("counts_exact") is not True:
                issues.append(prefix + "inexact_epoch")
        fields = ("kernel_launches", "sfu_instructions", "operations") + (("reference_loop_slots",) if reference else ())
        for name in fields:
            values = [integral(name, epoch) for epoch in epochs if isinstance(epoch, dict)]
            agree("epoch_total_" + name, sum(values) if all(v is not None for v in values) else None, integral(name))
    sanity = benchmark.get("sanity") or {}
    if sanity.get("finite_output_sample") is False:
        issues.append(prefix + "output_sanity_failed")
    if not reference:
        if sanity.get("numerical_validation_passed") is not True:
            issues.append("sfu_numerical_validation_failed_or_missing")
        checked = (benchmark.get("numerical_validation") or {}).get("checked_values")
        if isinstance(checked, bool) or not isinstance(checked, (int, float)) or not math.isfinite(checked) or checked <= 0:
            issues.append("sfu_missing_one_step_reference_checks")
    return sorted(set(issues))


def memory_count_issues(benchmark, workload) -> list[str]:
    if workload not in ("l1", "l2", "hbm") or benchmark.get("kernel_implementation_version") not in MEMORY_VERSIONS:
        return []
    version, access = benchmark["kernel_implementation_version"], benchmark.get("access")
    read = version in MEMORY_SINGLE_STREAM_READ_VERSIONS
    factor = 1 if read else 4
    issues = []
    if access not in (("read",) if read else ("write", "copy")):
        issues.append("memory_contract_access_implementation_mismatch")
    if _number(benchmark.get("memory_accesses_per_thread_iteration")) != factor:
        issues.append("memory_contract_accesses_per_iteration_mismatch")
    threads, iterations = (_number(benchmark.get(k)) for k in ("threads", "iterations_per_launch"))
    if any(v is None or v <= 0 or not v.is_integer() for v in (threads, iterations)):
        issues.append("memory_contract_invalid_execution_parameters")
        return issues
    rows = [("total", benchmark)]
    epochs = benchmark.get("measure_epochs", benchmark.get("work_epochs"))
    if isinstance(epochs, list):
        rows.extend(("epoch_" + str(i), e) for i, e in enumerate(epochs) if isinstance(e, dict))
    for label, row in rows:
        admitted = _number(row.get("admitted_blocks"))
        if admitted is None or admitted < 0 or not admitted.is_integer():
            issues.append("memory_contract_missing_or_invalid_admissions:" + label)
            continue
        operations = admitted * threads * iterations * factor
        logical_bytes = operations * 4 * (2 if access == "copy" else 1)
        for name, expected in (("operations", operations), ("logical_bytes", logical_bytes)):
            actual = _number(row.get(name))
            if actual is None or actual < 0 or abs(actual - expected) > max(1.0, abs(expected) * 1e-6):
                issues.append("memory_contract_count_disagreement:" + label + ":" + name)
    return issues


NONLINEAR_ROW_WORKLOADS = {"rmsnorm", "softmax"}
NONLINEAR_STREAMING_MATH = "cuda_fp32_standard_streaming_v1"
NONLINEAR_Q_GRID_MATH = "cuda_fp32_q_grid_v2"
NONLINEAR_Q_GRID_VERSION = "fp32_complete_nonlinear_q_grid_v2"
NONLINEAR_COUNT_SOURCE = "synchronized_completed_launches"
RMS_EPSILON = 1e-5


def nonlinear_bytes_per_element(workload) -> int:
    """Logical bytes of one output element: RMSNorm reads x twice, gamma once and writes y;
    softmax reads x three times and writes y (nonlinear.py:17-19)."""
    return 16 if workload in NONLINEAR_ROW_WORKLOADS else 8


def nonlinear_count_issues(benchmark, workload) -> list[str]:
    """Denominator checks of a complete-nonlinear-function record (nonlinear.py:22-128).

    An element is one output value (a whole row reduction included for RMSNorm
    and softmax).  Q-grid records (cuda_fp32_q_grid_v2) must account for every
    completed launch: launches x Q x iterations elements, launches x blocks
    CTAs, per epoch and in total; older records are checked per admitted block.
    """
    if workload not in NONLINEAR_WORKLOADS:
        return []
    row = workload in NONLINEAR_ROW_WORKLOADS
    per_element = nonlinear_bytes_per_element(workload)
    issues: list[str] = []

    def count(key, obj=benchmark):
        v = obj.get(key)
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v) or v < 0 or v != int(v):
            issues.append("invalid_nonlinear_count:" + key)
            return None
        return v

    def agree(name, actual, expected):
        if actual is None or expected is None or not math.isclose(actual, expected, rel_tol=1e-9, abs_tol=1e-6):
            issues.append("nonlinear_count_disagreement:" + name)

    def times(*values):
        out = 1
        for v in values:
            if v is None:
                return None
            out *= v
        return out

    elements, operations = count("elements"), count("operations")
    if elements is not None and elements <= 0:
        issues.append("missing_nonlinear_elements")
    agree("operations_are_elements", operations, elements)
    agree("logical_bytes", count("logical_bytes"), times(elements, per_element))
    width = count("row_width")
    if row:
        if width is None or not 1 <= width <= 65536 or width != int(width):
            issues.append("invalid_nonlinear_row_width")
        agree("row_evaluations", count("row_evaluations"), elements / width if elements is not None and width else None)
    else:
        agree("row_width", width, 0)
        agree("row_evaluations", count("row_evaluations"), 0)
    blocks, ws, iterations, admitted = (count(k) for k in ("blocks", "working_set_bytes", "iterations_per_launch",
                                                             "admitted_blocks"))
    math_tag, version = benchmark.get("math_implementation"), benchmark.get("kernel_implementation_version")
    q_grid = math_tag == NONLINEAR_Q_GRID_MATH or version == NONLINEAR_Q_GRID_VERSION
    launches = batch_launches = q = None
    if q_grid:
        if math_tag != NONLINEAR_Q_GRID_MATH or version != NONLINEAR_Q_GRID_VERSION:
            issues.append("unsupported_nonlinear_q_grid_implementation")
        if benchmark.get("block_completion_count_source") != NONLINEAR_COUNT_SOURCE:
            issues.append("unsupported_nonlinear_block_completion_count_source")
        q, threads, launches = count("input_elements"), count("threads"), count("kernel_launches")
        if "batch_launches" in benchmark:
            batch_launches = count("batch_launches")
            if not batch_launches:
                issues.append("invalid_nonlinear_batch_launches")
        if "batches" in benchmark:
            agree("completed_batch_kernel_launches", launches, times(count("batches"), batch_launches))
        if ws is None or ws <= 0 or ws % 4:
            issues.append("invalid_nonlinear_input_word_alignment")
        agree("input_elements", q, ws / 4 if ws is not None else None)
        if q is None or q <= 0 or (width and row and q % width):
            issues.append("incomplete_nonlinear_input_or_row")
        if threads is None or not 32 <= threads <= 1024 or threads % 32:
            issues.append("invalid_nonlinear_threads")
        mode = benchmark.get("grid_mode")
        if mode not in ("auto", "fixed"):
            issues.append("invalid_nonlinear_grid_mode")
        elif mode == "auto" and q and threads and (not row or width):
            agree("auto_grid_blocks", blocks, q / width if row else math.ceil(q / threads))
        if not blocks or blocks > 1000000 or not iterations or not launches:
            issues.append("missing_nonlinear_execution_counts")
        if launches is not None and blocks is not None:
            agree("completed_launch_admissions", admitted, launches * blocks)
        agree("completed_launch_elements", elements, times(launches, q, iterations))
    elif blocks and ws and iterations and admitted:
        # Contiguous per-CTA slices of the first streaming implementation.
        agree("admission_elements", elements, admitted * (ws / 4 / blocks) * iterations)
        if ws % (4 * blocks * (width if row and width else 1)):
            issues.append("incomplete_nonlinear_block_slice_or_row")
    else:
        issues.append("missing_nonlinear_execution_counts")
    if math_tag not in (NONLINEAR_STREAMING_MATH, NONLINEAR_Q_GRID_MATH) or benchmark.get("input_precision") != "fp32":
        issues.append("unsupported_nonlinear_math_contract")
    if workload == "rmsnorm" and (benchmark.get("rms_epsilon") != RMS_EPSILON or benchmark.get("affine_gamma") is not True):
        issues.append("unsupported_rmsnorm_definition")
    if (benchmark.get("sanity") or {}).get("numerical_validation_passed") is not True:
        issues.append("nonlinear_numerical_validation_failed_or_missing")
    checked = (benchmark.get("numerical_validation") or {}).get("checked_values")
    if isinstance(checked, bool) or not isinstance(checked, (int, float)) or not math.isfinite(checked) or checked <= 0:
        issues.append("missing_nonlinear_numerical_reference_checks")
    epochs = benchmark.get("measure_epochs")
    if not isinstance(epochs, list) or not epochs:
        issues.append("missing_nonlinear_measure_epochs")
        return sorted(set(issues))
    for epoch in epochs:
        if not isinstance(epoch, dict):
            issues.append("invalid_nonlinear_epoch")
            continue
        e = count("elements", epoch)
        agree("epoch_operations_are_elements", count("operations", epoch), e)
        agree("epoch_logical_bytes", count("logical_bytes", epoch), times(e, per_element))
        agree("epoch_rows", count("row_evaluations", epoch), e / width if e is not None and width and row else 0)
        if q_grid:
            epoch_launches = count("kernel_launches", epoch)
            if "batches" in epoch:
                agree("epoch_completed_batch_kernel_launches", epoch_launches, times(count("batches", epoch), batch_launches))
            agree("epoch_completed_launch_admissions", count("admitted_blocks", epoch), times(epoch_launches, blocks))
            agree("epoch_completed_launch_elements", e, times(epoch_launches, q, iterations))
        if epoch.get("counts_exact") is not True:
            issues.append("inexact_nonlinear_measure_epoch")

    def total(key):
        return sum(ep.get(key, 0) for ep in epochs if isinstance(ep, dict) and isinstance(ep.get(key), (int, float)))
    agree("epoch_total_elements", total("elements"), elements)
    if q_grid:
        agree("epoch_total_kernel_launches", total("kernel_launches"), launches)
    return sorted(set(issues))
