"""Deterministic benchmark records for the SFU and memory count contracts.

``sfu_cases()`` yields (name, workload, reference, record): consistent SFU
treatment records (powerbench ``result``) and paired active-reference
records (``active_reference_result``) for every opcode, then one change at a
time that a rule must catch or accept.  ``memory_cases()`` yields (name,
workload, record) for the scalar read and the four-stream write/copy
implementations.  tests/golden/make_contract_golden.py runs the reference's
sfu.count_issues (sfu.py:23-115) and memory.count_issues (memory.py:114-144)
on them; tests/test_contracts.py checks powermodeling_b200.contracts.
"""
from __future__ import annotations

import copy

from nonlinear_cases import _DROP, _add, _scale, _set

OPCODES = ("ex2", "lg2", "rcp", "rsqrt", "sqrt", "tanh")


def sfu_record(primitive: str, *, reference: bool = False, lanes: int = 8192, threads: int = 256, chains: int = 4,
               iterations: int = 64, batch_launches: int = 2, epoch_batches: tuple = (2, 1), grid_mode: str = "auto",
               blocks: int | None = None) -> dict:
    if grid_mode == "auto":
        blocks = -(-lanes // threads)
    slots_per_launch = lanes * iterations * chains
    epochs = []
    for b in epoch_batches:
        launches = b * batch_launches
        work = 0 if reference else launches * slots_per_launch
        epoch = {"batches": b, "kernel_launches": launches, "admitted_blocks": launches * blocks,
                 "sfu_instructions": work, "operations": work, "logical_bytes": 0, "elements": 0,
                 "counts_exact": True, "sfu_lanes": lanes, "sfu_chains": chains, "batch_launches": batch_launches}
        if reference:
            epoch["reference_loop_slots"] = launches * slots_per_launch
        epochs.append(epoch)
    batches = sum(epoch_batches)
    launches = batches * batch_launches
    work = 0 if reference else launches * slots_per_launch
    rec = {"type": "active_reference_result" if reference else "result",
           "workload": "control" if reference else "sfu_" + primitive,
           "kernel_implementation_version": "sfu_register_control_v1" if reference else "sfu_register_recurrence_v1",
           "math_implementation": "ptx_approx_register_v1",
           "sfu_input_policy": "feedback_xor_iteration_mantissa_0p5_1_v1", "sfu_primitive": primitive,
           "sfu_ptx_opcode": primitive + (".approx.f32" if primitive == "tanh" else ".approx.ftz.f32"),
           "sfu_approximate": True, "sfu_flush_to_zero": primitive != "tanh",
           "sfu_exponent_base": 2 if primitive in ("ex2", "lg2") else None,
           "block_completion_count_source": "synchronized_completed_launches",
           "sfu_lanes": lanes, "sfu_chains": chains, "iterations_per_launch": iterations, "blocks": blocks,
           "threads": threads, "grid_mode": grid_mode, "batch_launches": batch_launches, "batches": batches,
           "kernel_launches": launches, "admitted_blocks": launches * blocks, "sfu_instructions": work,
           "operations": work, "logical_bytes": 0, "elements": 0,
           "sanity": {"finite_output_sample": True, "numerical_validation_passed": True},
           "numerical_validation": {"checked_values": 16}, "measure_epochs": epochs}
    if reference:
        rec["reference_kind"] = "register_loop_without_sfu"
        rec["reference_loop_slots"] = launches * slots_per_launch
    return rec


SFU_CHANGES = (
    ("version_other", _set(("kernel_implementation_version",), "sfu_register_recurrence_v0")),
    ("math_other", _set(("math_implementation",), "libm")),
    ("policy_other", _set(("sfu_input_policy",), "uniform")),
    ("primitive_other", _set(("sfu_primitive",), "exp")),
    ("opcode_other", _set(("sfu_ptx_opcode",), "ex2.f32")),
    ("approximate_one", _set(("sfu_approximate",), 1)),
    ("ftz_flipped", lambda rec: (rec.__setitem__("sfu_flush_to_zero", not rec["sfu_flush_to_zero"]), rec)[1]),
    ("base_ten", _set(("sfu_exponent_base",), 10)),
    ("base_float_two", lambda rec: (rec.__setitem__("sfu_exponent_base", 2.0 if rec["sfu_exponent_base"] else None), rec)[1]),
    ("count_source_atomics", _set(("block_completion_count_source",), "per_sm_admission_atomics")),
    ("workload_other", _set(("workload",), "sfu_ex2")),
    ("reference_kind_other", _set(("reference_kind",), "issue_loop")),
    ("lanes_zero", _set(("sfu_lanes",), 0)),
    ("lanes_fraction", _set(("sfu_lanes",), 8192.5)),
    ("lanes_bool", _set(("sfu_lanes",), True)),
    ("chains_two", _set(("sfu_chains",), 2)),
    ("chains_missing", _set(("sfu_chains",), _DROP)),
    ("iterations_zero", _set(("iterations_per_launch",), 0)),
    ("iterations_huge", _set(("iterations_per_launch",), 2 ** 33)),
    ("blocks_huge", _set(("blocks",), 2000000)),
    ("blocks_plus_one", _add("blocks", 1)),
    ("threads_100", _set(("threads",), 100)),
    ("threads_16", _set(("threads",), 16)),
    ("threads_missing", _set(("threads",), _DROP)),
    ("launches_zero", _set(("kernel_launches",), 0)),
    ("launches_plus_one", _add("kernel_launches", 1)),
    ("grid_mode_guess", _set(("grid_mode",), "guess")),
    ("grid_mode_fixed", _set(("grid_mode",), "fixed")),
    ("batch_launches_zero", _set(("batch_launches",), 0)),
    ("batch_launches_huge", _set(("batch_launches",), 70000)),
    ("batch_launches_missing", _set(("batch_launches",), _DROP)),
    ("batches_missing", _set(("batches",), _DROP)),
    ("batches_plus_one", _add("batches", 1)),
    ("admitted_plus_one", _add("admitted_blocks", 1)),
    ("instructions_plus_one", _add("sfu_instructions", 1)),
    ("operations_doubled", _scale("operations", 2)),
    ("operations_nan", _set(("operations",), float("nan"))),
    ("logical_bytes_one", _set(("logical_bytes",), 1)),
    ("elements_missing", _set(("elements",), _DROP)),
    ("slots_plus_one", lambda rec: (rec.__setitem__("reference_loop_slots", rec.get("reference_loop_slots", 0) + 1), rec)[1]),
    ("epochs_empty", _set(("measure_epochs",), [])),
    ("epochs_missing", _set(("measure_epochs",), _DROP)),
    ("epoch_not_dict", lambda rec: (rec["measure_epochs"].append("x"), rec)[1]),
    ("epoch_inexact", _set(("measure_epochs", 0, "counts_exact"), False)),
    ("epoch_lanes_other", _set(("measure_epochs", 1, "sfu_lanes"), 4096)),
    ("epoch_batch_launches_other", _set(("measure_epochs", 0, "batch_launches"), 3)),
    ("epoch_launches_plus_one", _add("kernel_launches", 1, epoch=0)),
    ("epoch_admitted_plus_one", _add("admitted_blocks", 1, epoch=1)),
    ("epoch_instructions_plus_one", _add("sfu_instructions", 1, epoch=0)),
    ("epoch_operations_negative", _set(("measure_epochs", 1, "operations"), -1)),
    ("epoch_batches_missing", _set(("measure_epochs", 0, "batches"), _DROP)),
    ("epoch_elements_one", _set(("measure_epochs", 0, "elements"), 1)),
    ("epoch_dropped", lambda rec: (rec["measure_epochs"].pop(), rec)[1]),
    ("output_not_finite", _set(("sanity", "finite_output_sample"), False)),
    ("validation_failed", _set(("sanity", "numerical_validation_passed"), False)),
    ("sanity_missing", _set(("sanity",), _DROP)),
    ("checked_zero", _set(("numerical_validation", "checked_values"), 0)),
    ("checked_bool", _set(("numerical_validation", "checked_values"), True)),
    ("validation_missing", _set(("numerical_validation",), _DROP)),
)


def sfu_cases():
    """(name, workload, reference, record) in a fixed order."""
    out = []
    for primitive in OPCODES:
        workload = "sfu_" + primitive
        for reference in (False, True):
            role = "reference" if reference else "treatment"
            bases = [("auto", sfu_record(primitive, reference=reference)),
                     ("fixed", sfu_record(primitive, reference=reference, grid_mode="fixed", blocks=148 * 2,
                                          lanes=148 * 2 * 256, chains=8)),
                     ("chains1_threads1024", sfu_record(primitive, reference=reference, chains=1, threads=1024))]
            for label, base in bases:
                out.append((f"{workload}/{role}/{label}", workload, reference, copy.deepcopy(base)))
            for name, change in SFU_CHANGES:
                out.append((f"{workload}/{role}/auto/{name}", workload, reference, change(copy.deepcopy(bases[0][1]))))
    out.append(("not_sfu", "hbm", False, sfu_record("ex2")))
    return out


def memory_record(access: str = "read", *, threads: int = 256, iterations: int = 128, admitted: int = 296,
                  epoch_admitted: tuple = (148, 148), epochs_key: str = "measure_epochs") -> dict:
    read = access == "read"
    factor = 1 if read else 4
    scale = 4 * (2 if access == "copy" else 1)

    def row(a):
        ops = a * threads * iterations * factor
        return {"admitted_blocks": a, "operations": ops, "logical_bytes": ops * scale}

    rec = {"type": "result", "workload": "hbm", "access": access,
           "kernel_implementation_version": "scalar_single_stream_read_v3" if read else "scalar_four_stream_write_copy_v1",
           "memory_accesses_per_thread_iteration": factor, "threads": threads, "iterations_per_launch": iterations,
           **row(admitted), epochs_key: [dict(row(a), counts_exact=True) for a in epoch_admitted]}
    return rec


MEMORY_CHANGES = (
    ("access_other", _set(("access",), "scan")),
    ("accesses_other", _set(("memory_accesses_per_thread_iteration",), 2)),
    ("accesses_missing", _set(("memory_accesses_per_thread_iteration",), _DROP)),
    ("threads_zero", _set(("threads",), 0)),
    ("threads_fraction", _set(("threads",), 256.5)),
    ("iterations_missing", _set(("iterations_per_launch",), _DROP)),
    ("admitted_missing", _set(("admitted_blocks",), _DROP)),
    ("admitted_negative", _set(("admitted_blocks",), -1)),
    ("admitted_fraction", _set(("admitted_blocks",), 1.5)),
    ("operations_plus_one", _add("operations", 1)),
    ("operations_plus_half_ppm", lambda rec: (rec.__setitem__("operations", rec["operations"] * (1 + 5e-7)), rec)[1]),
    ("operations_plus_two_ppm", lambda rec: (rec.__setitem__("operations", rec["operations"] * (1 + 2e-6)), rec)[1]),
    ("operations_negative", _set(("operations",), -4)),
    ("logical_bytes_halved", _scale("logical_bytes", 0.5)),
    ("logical_bytes_bool", _set(("logical_bytes",), True)),
    ("epoch_admitted_plus_one", lambda rec: (rec["measure_epochs"][0].__setitem__("admitted_blocks", 149), rec)[1]
     if "measure_epochs" in rec else rec),
    ("epoch_not_dict", lambda rec: (rec.get("measure_epochs", rec.get("work_epochs")).append(3), rec)[1]),
    ("epochs_not_list", _set(("measure_epochs",), "none")),
    ("version_other", _set(("kernel_implementation_version",), "vector_read_v1")),
)


def memory_cases():
    """(name, workload, record) in a fixed order."""
    out = []
    for access in ("read", "write", "copy"):
        for workload in (("l1", "l2", "hbm") if access == "read" else ("hbm",)):
            base = memory_record(access)
            base["workload"] = workload
            out.append((f"{workload}/{access}", workload, copy.deepcopy(base)))
            for name, change in MEMORY_CHANGES:
                out.append((f"{workload}/{access}/{name}", workload, change(copy.deepcopy(base))))
    work = memory_record("read", epochs_key="work_epochs")
    out.append(("hbm/read/work_epochs", "hbm", copy.deepcopy(work)))
    v2 = memory_record("read")
    v2["kernel_implementation_version"] = "scalar_single_stream_read_v2"
    out.append(("hbm/read/v2", "hbm", v2))
    out.append(("not_memory", "tensor", memory_record("read")))
    return out
