"""Deterministic benchmark records for the nonlinear count contract (nonlinear.py:22-128).

``cases()`` yields (name, workload, record): a consistent Q-grid result for
each function and grid mode, then one change at a time that a count rule
must catch (or must accept), plus records of the first streaming
implementation.  tests/golden/make_nonlinear_golden.py runs the reference's
count_issues on them; tests/test_nonlinear.py checks the restatement.
"""
from __future__ import annotations

import copy

FUNCTIONS = ("exp", "tanh", "silu", "softmax", "rmsnorm")
ROWS = ("softmax", "rmsnorm")


def q_grid_record(workload: str, *, q: int = 4128, threads: int = 96, width: int | None = None, grid_mode: str = "auto",
                  blocks: int | None = None, iterations: int = 2, batch_launches: int = 3,
                  epoch_batches: tuple = (2, 3)) -> dict:
    row = workload in ROWS
    width = (width or 129) if row else 0
    if row:
        q = q // width * width
    if grid_mode == "auto":
        blocks = q // width if row else -(-q // threads)
    per_element = 16 if row else 8
    epochs = []
    for b in epoch_batches:
        launches = b * batch_launches
        el = launches * q * iterations
        epochs.append({"batches": b, "kernel_launches": launches, "admitted_blocks": launches * blocks,
                       "operations": el, "logical_bytes": el * per_element, "elements": el,
                       "row_evaluations": el // width if row else 0, "counts_exact": True, "counter_readback_ns": 0})
    batches = sum(epoch_batches)
    launches = batches * batch_launches
    elements = launches * q * iterations
    rec = {"type": "result", "workload": workload, "batches": batches, "batch_launches": batch_launches,
           "kernel_launches": launches, "iterations_per_launch": iterations, "blocks": blocks, "threads": threads,
           "admitted_blocks": launches * blocks, "working_set_bytes": q * 4, "input_elements": q,
           "grid_mode": grid_mode, "kernel_implementation_version": "fp32_complete_nonlinear_q_grid_v2",
           "math_implementation": "cuda_fp32_q_grid_v2", "block_completion_count_source": "synchronized_completed_launches",
           "operations": elements, "logical_bytes": elements * per_element, "elements": elements,
           "row_width": width, "row_evaluations": elements // width if row else 0,
           "rms_epsilon": 1e-05 if workload == "rmsnorm" else None, "affine_gamma": workload == "rmsnorm",
           "input_precision": "fp32", "numerical_validation": {"checked_values": 16},
           "sanity": {"numerical_validation_passed": True}, "measure_epochs": epochs}
    return rec


def streaming_v1_record(workload: str, *, blocks: int = 4, slice_elements: int = 1032, iterations: int = 3,
                        admitted: int = 40) -> dict:
    """A record of the first streaming implementation: contiguous per-CTA slices, admission counts."""
    row = workload in ROWS
    width = 129 if row else 0
    if row:
        slice_elements = slice_elements // width * width
    ws = blocks * slice_elements * 4
    elements = admitted * slice_elements * iterations
    per_element = 16 if row else 8
    return {"type": "result", "workload": workload, "blocks": blocks, "threads": 256, "iterations_per_launch": iterations,
            "admitted_blocks": admitted, "working_set_bytes": ws, "math_implementation": "cuda_fp32_standard_streaming_v1",
            "kernel_implementation_version": "fp32_complete_nonlinear_v1",
            "operations": elements, "logical_bytes": elements * per_element, "elements": elements,
            "row_width": width, "row_evaluations": elements // width if row else 0,
            "rms_epsilon": 1e-05 if workload == "rmsnorm" else None, "affine_gamma": workload == "rmsnorm",
            "input_precision": "fp32", "numerical_validation": {"checked_values": 8},
            "sanity": {"numerical_validation_passed": True},
            "measure_epochs": [{"operations": elements, "logical_bytes": elements * per_element, "elements": elements,
                                "row_evaluations": elements // width if row else 0, "counts_exact": True}]}


def _set(path, value):
    def change(rec):
        obj = rec
        for key in path[:-1]:
            obj = obj[key]
        if value is _DROP:
            obj.pop(path[-1], None)
        else:
            obj[path[-1]] = value
        return rec
    return change


_DROP = object()


def _scale(key, factor):
    def change(rec):
        rec[key] = rec[key] * factor
        return rec
    return change


def _add(key, delta, epoch=None):
    def change(rec):
        obj = rec if epoch is None else rec["measure_epochs"][epoch]
        obj[key] = obj[key] + delta
        return rec
    return change


CHANGES = (
    ("elements_plus_one", _add("elements", 1)),
    ("operations_plus_one", _add("operations", 1)),
    ("logical_bytes_halved", _scale("logical_bytes", 0.5)),
    ("elements_bool", _set(("elements",), True)),
    ("elements_negative", _set(("elements",), -8)),
    ("elements_nan", _set(("elements",), float("nan"))),
    ("elements_fraction", _set(("elements",), 10.5)),
    ("elements_zero", _set(("elements",), 0)),
    ("row_width_zero", _set(("row_width",), 0)),
    ("row_width_large", _set(("row_width",), 70000)),
    ("row_width_fraction", _set(("row_width",), 129.5)),
    ("row_width_missing", _set(("row_width",), _DROP)),
    ("row_evaluations_plus_one", _add("row_evaluations", 1)),
    ("blocks_plus_one", _add("blocks", 1)),
    ("blocks_zero", _set(("blocks",), 0)),
    ("blocks_huge", _set(("blocks",), 2000000)),
    ("admitted_plus_one", _add("admitted_blocks", 1)),
    ("working_set_unaligned", _add("working_set_bytes", 2)),
    ("working_set_partial_row", _add("working_set_bytes", 4)),
    ("input_elements_plus_one", _add("input_elements", 1)),
    ("input_elements_missing", _set(("input_elements",), _DROP)),
    ("threads_100", _set(("threads",), 100)),
    ("threads_2048", _set(("threads",), 2048)),
    ("threads_missing", _set(("threads",), _DROP)),
    ("kernel_launches_plus_one", _add("kernel_launches", 1)),
    ("batch_launches_zero", _set(("batch_launches",), 0)),
    ("batch_launches_missing", _set(("batch_launches",), _DROP)),
    ("batches_missing", _set(("batches",), _DROP)),
    ("batches_plus_one", _add("batches", 1)),
    ("grid_mode_guess", _set(("grid_mode",), "guess")),
    ("grid_mode_fixed", _set(("grid_mode",), "fixed")),
    ("iterations_zero", _set(("iterations_per_launch",), 0)),
    ("math_v1_with_q_grid_version", _set(("math_implementation",), "cuda_fp32_standard_streaming_v1")),
    ("version_other", _set(("kernel_implementation_version",), "fp32_complete_nonlinear_v1")),
    ("math_unknown", _set(("math_implementation",), "libm")),
    ("count_source_atomics", _set(("block_completion_count_source",), "per_sm_admission_atomics")),
    ("input_fp16", _set(("input_precision",), "fp16")),
    ("rms_epsilon_other", _set(("rms_epsilon",), 1e-6)),
    ("affine_gamma_false", _set(("affine_gamma",), False)),
    ("validation_failed", _set(("sanity", "numerical_validation_passed"), False)),
    ("sanity_missing", _set(("sanity",), _DROP)),
    ("checked_zero", _set(("numerical_validation", "checked_values"), 0)),
    ("checked_bool", _set(("numerical_validation", "checked_values"), True)),
    ("epochs_empty", _set(("measure_epochs",), [])),
    ("epochs_not_list", _set(("measure_epochs",), {"elements": 1})),
    ("epoch_not_dict", lambda rec: (rec["measure_epochs"].append(7), rec)[1]),
    ("epoch_inexact", _set(("measure_epochs", 0, "counts_exact"), False)),
    ("epoch_elements_plus_one", _add("elements", 1, epoch=0)),
    ("epoch_operations_plus_one", _add("operations", 1, epoch=1)),
    ("epoch_logical_bytes_plus_one", _add("logical_bytes", 1, epoch=0)),
    ("epoch_rows_plus_one", _add("row_evaluations", 1, epoch=1)),
    ("epoch_admitted_plus_one", _add("admitted_blocks", 1, epoch=0)),
    ("epoch_launches_plus_one", _add("kernel_launches", 1, epoch=1)),
    ("epoch_batches_plus_one", _add("batches", 1, epoch=0)),
    ("epoch_batches_missing", _set(("measure_epochs", 0, "batches"), _DROP)),
    ("epoch_elements_bool", _set(("measure_epochs", 1, "elements"), False)),
    ("epoch_dropped", lambda rec: (rec["measure_epochs"].pop(), rec)[1]),
)


def cases():
    """(name, workload, record) in a fixed order."""
    out = []
    for workload in FUNCTIONS:
        bases = [("auto", q_grid_record(workload)),
                 ("fixed3", q_grid_record(workload, grid_mode="fixed", blocks=3)),
                 ("auto_threads1024", q_grid_record(workload, threads=1024, q=8192)),
                 ("fixed_width1024", q_grid_record(workload, grid_mode="fixed", blocks=2, width=1024, q=5 * 1024))]
        for label, base in bases:
            out.append((f"{workload}/{label}", workload, copy.deepcopy(base)))
        for name, change in CHANGES:
            out.append((f"{workload}/auto/{name}", workload, change(copy.deepcopy(bases[0][1]))))
        v1 = streaming_v1_record(workload)
        out.append((f"{workload}/v1", workload, copy.deepcopy(v1)))
        for name, change in (("admitted_zero", _set(("admitted_blocks",), 0)),
                             ("elements_plus_one", _add("elements", 1)),
                             ("slice_partial", _add("working_set_bytes", 4)),
                             ("epoch_inexact", _set(("measure_epochs", 0, "counts_exact"), False))):
            out.append((f"{workload}/v1/{name}", workload, change(copy.deepcopy(v1))))
    out.append(("not_nonlinear", "hbm", q_grid_record("exp")))
    return out
