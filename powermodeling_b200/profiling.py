"""Nsight Compute evidence for this engine's kernels: the counter list, the
ncu command for one powerbench trial, and the raw-CSV reader with unit
normalisation (the reference's profiling.py:24-149).

The reader keeps every launch's raw value beside its number in base units and
never fills a gap: an unknown unit, an ambiguous number (a comma decimal, an
instance list, ``N/A``) or a non-finite value is kept as an error.  Nsight's
K/M/G byte prefixes are decimal; KiB/MiB/GiB are binary.

The admission rules that turn these rows into a verified target
(validation.assess_profile / validate_evidence) are not provided here; a
trial record that carries profiler evidence is refused by the analysis.
"""
from __future__ import annotations

import csv
import io
import math
import re
from typing import Any, Iterable

# Counter names (validation.py:53-66), in the reference's request order.
LOCAL_LOAD = "l1tex__t_sectors_pipe_lsu_mem_local_op_ld.sum"
LOCAL_STORE = "l1tex__t_sectors_pipe_lsu_mem_local_op_st.sum"
DRAM_READ = "dram__bytes_read.sum"
DRAM_WRITE = "dram__bytes_write.sum"
DURATION = "gpu__time_duration.sum"
SM_HZ = "sm__cycles_elapsed.avg.per_second"
L1_SECTORS = "l1tex__t_sectors_pipe_lsu_mem_global_op_ld.sum"
L1_HITS = "l1tex__t_sectors_pipe_lsu_mem_global_op_ld_lookup_hit.sum"
L1_MISSES = "l1tex__t_sectors_pipe_lsu_mem_global_op_ld_lookup_miss.sum"
L1_REQUESTS = "l1tex__t_requests_pipe_lsu_mem_global_op_ld.sum"
L2_READ = "lts__t_sectors_srcunit_tex_op_read.sum"
L2_READ_HITS = "lts__t_sectors_srcunit_tex_op_read_lookup_hit.sum"
L2_WRITE = "lts__t_sectors_srcunit_tex_op_write.sum"
TENSOR_INSTRUCTIONS = ("sm__inst_executed_pipe_tensor.sum", "smsp__inst_executed_pipe_tensor.sum")
TENSOR_ACTIVITY = ("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
                   "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active")
SFU_INSTRUCTIONS = ("smsp__inst_executed_pipe_sfu.sum", "sm__inst_executed_pipe_sfu.sum")
SFU_ACTIVITY = ("sm__pipe_sfu_cycles_active.avg.pct_of_peak_sustained_elapsed",
                "smsp__pipe_sfu_cycles_active.avg.pct_of_peak_sustained_elapsed",
                "sm__pipe_sfu_cycles_active.avg.pct_of_peak_sustained_active",
                "smsp__pipe_sfu_cycles_active.avg.pct_of_peak_sustained_active")
READ_OVERHEAD = ("smsp__sass_thread_inst_executed_op_global_ld_pred_on.sum",
                 "smsp__sass_thread_inst_executed_op_integer_pred_on.sum")
METRICS = list(dict.fromkeys([
    DRAM_READ, DRAM_WRITE, DURATION, SM_HZ, "dram__cycles_elapsed.avg.per_second", L2_READ, L2_READ_HITS, L2_WRITE,
    L1_SECTORS, L1_HITS, L1_MISSES, L1_REQUESTS, LOCAL_LOAD, LOCAL_STORE, *TENSOR_INSTRUCTIONS, *TENSOR_ACTIVITY,
    *SFU_INSTRUCTIONS, *SFU_ACTIVITY, *READ_OVERHEAD,
    "dram__throughput.avg.pct_of_peak_sustained_elapsed", "lts__throughput.avg.pct_of_peak_sustained_elapsed",
    "l1tex__throughput.avg.pct_of_peak_sustained_elapsed", "sm__warps_active.avg.pct_of_peak_sustained_active",
    "sm__warps_active.avg.pct_of_peak_sustained_elapsed", "lts__t_sector_hit_rate.pct", "l1tex__t_sector_hit_rate.pct"]))

# This engine's measured kernels (the fills, checks and the cuBLAS arm's library kernels excluded).
TARGET_KERNELS = ("read_scalar_kernel", "read_vector_kernel", "write_copy_scalar_kernel", "copy_vector_kernel",
                  "chase_words_kernel", "chase_lines_kernel", "control_kernel", "tensor_mma_kernel", "sfu_kernel",
                  "pointwise_stream_kernel", "row_stream_kernel", "row_warp_kernel", "row_cta_kernel")


def available_metric_names(text) -> set:
    """Counter names in ncu --query-metrics output (or a given collection)."""
    if isinstance(text, (set, list, tuple)):
        return set(text)
    return set(re.findall(r"\b[a-zA-Z][a-zA-Z0-9_]*__[a-zA-Z0-9_.]+", text or ""))


def profile_command(ncu: str, powerbench_argv: list, workload: str, device_index: int = 0, available=None,
                    log_file=None, report_path=None) -> list[str]:
    """The ncu command that captures the counters of one powerbench trial's measured kernel:
    raw page, base units, no clock or cache control, application replay from the profiler start
    the engine places around its measured phase, and for every workload but the GEMM arm one
    launch of this engine's target kernel."""
    advertised = available_metric_names(available) if available is not None else set(METRICS)
    metrics = [m for m in METRICS if m in advertised]
    if not metrics:
        raise ValueError("None of the validation counters are available")
    command = [ncu, "--devices", str(device_index), "--csv", "--print-units", "base", "--page", "raw",
               "--target-processes", "all", "--clock-control", "none", "--cache-control", "none",
               "--replay-mode", "application", "--profile-from-start", "off", "--metrics", ",".join(metrics)]
    if log_file is not None:
        command += ["--log-file", str(log_file)]
    if report_path is not None:
        command += ["--export", str(report_path), "--force-overwrite"]
    if workload != "gemm":
        command += ["--kernel-name", "regex:.*(" + "|".join(TARGET_KERNELS) + ").*", "--launch-count", "1"]
    return command + [str(a) for a in powerbench_argv]


# ---------------------------------------------------------------------------- units
_PLAIN = re.compile(r"^[+-]?(?:\d+(?:\.\d*)?|\.\d+)(?:[eE][+-]?\d+)?$")
_GROUPED = (re.compile(r"^[+-]?\d{1,3}(?:,\d{3})+(?:\.\d+)?(?:[eE][+-]?\d+)?$"), ","),
_GROUPED += ((re.compile(r"^[+-]?\d{1,3}(?: \d{3})+(?:\.\d+)?(?:[eE][+-]?\d+)?$"), " "),)

# unit text -> (factor to the base unit, base unit)
_SCALE: dict[str, tuple[float, str]] = {"": (1, "count"), "count": (1, "count"), "%": (1, "%"), "percent": (1, "%")}
for _names, _factor, _base in (
        (("byte", "bytes", "B"), 1, "byte"), (("Kbyte", "KB"), 1e3, "byte"), (("Mbyte", "MB"), 1e6, "byte"),
        (("Gbyte", "GB"), 1e9, "byte"), (("KiB",), 1024, "byte"), (("MiB",), 1024 ** 2, "byte"),
        (("GiB",), 1024 ** 3, "byte"),
        (("second", "s"), 1, "second"), (("msecond", "ms"), 1e-3, "second"),
        (("usecond", "us", "microsecond"), 1e-6, "second"), (("nsecond", "ns", "nanosecond"), 1e-9, "second"),
        (("cycle/second", "cycle/s", "Hz"), 1, "cycle/second"), (("KHz",), 1e3, "cycle/second"),
        (("MHz",), 1e6, "cycle/second"), (("GHz",), 1e9, "cycle/second"),
        (("cycle/nsecond",), 1e9, "cycle/second"), (("cycle/usecond",), 1e6, "cycle/second"),
        (("sector",), 1, "sector"), (("request",), 1, "request"), (("inst", "instruction"), 1, "inst"),
        (("cycle",), 1, "cycle")):
    for _name in _names:
        _SCALE[_name] = (_factor, _base)


def _unit(text: str):
    """(factor, base) of a unit, a per-second rate of a known unit included, else None."""
    if text in _SCALE:
        return _SCALE[text]
    for suffix in ("/second", "/s"):
        if text.endswith(suffix) and text[:-len(suffix)] in _SCALE:
            factor, base = _SCALE[text[:-len(suffix)]]
            return factor, base + "/second"
    return None


def normalize_metric_value(value, unit) -> tuple[float | None, str | None, str | None]:
    """(number in base units, base unit, error) of one raw counter cell; never zero-filled."""
    if value is None or isinstance(value, bool):
        return None, None, "missing_or_non_numeric_counter"
    raw = str(value).strip().replace("\u00a0", " ").replace("\u202f", " ")
    if raw.endswith("%") and str(unit).strip() in ("%", "percent"):
        raw = raw[:-1].strip()
    for pattern, separator in _GROUPED:
        if pattern.fullmatch(raw):
            raw = raw.replace(separator, "")
            break
    if not _PLAIN.fullmatch(raw):
        return None, None, "missing_or_ambiguous_counter"
    number = float(raw)
    if not math.isfinite(number):
        return None, None, "non_finite_counter"
    text = str(unit or "").strip().replace("µ", "u").replace("μ", "u")
    scale = _unit(text)
    if scale is None:
        return None, text, "unsupported_counter_unit"
    factor, base = scale
    scaled = number * factor
    return (scaled, base, None) if math.isfinite(scaled) else (None, base, "non_finite_counter")


def parse_ncu_csv(text: str) -> list[dict[str, Any]]:
    """One row per (launch, counter) of an ncu --csv --page raw log: raw value and unit kept,
    the base-unit number and any parse error beside them."""
    lines = text.splitlines()
    header = next((i for i, line in enumerate(lines) if "Metric Name" in line and "Metric Value" in line), None)
    if header is None:
        raise ValueError("Nsight CSV missing Metric Name/Metric Value header")
    rows = []
    for row in csv.DictReader(io.StringIO("\n".join(lines[header:]))):
        metric, value = row.get("Metric Name"), row.get("Metric Value")
        if not metric or metric == "Metric Name":
            continue
        number, base, error = normalize_metric_value(value, row.get("Metric Unit"))
        rows.append({"id": row.get("ID"), "kernel": row.get("Kernel Name"), "device": row.get("Device"),
                     "metric": metric, "unit": row.get("Metric Unit"), "value": value,
                     "numeric_value": number, "normalized_unit": base, "parse_error": error})
    if not rows:
        raise ValueError("Nsight CSV contained no counter values")
    return rows


def launch_counters(rows: Iterable[dict]) -> dict[tuple, dict[str, float | None]]:
    """Per (launch id, kernel): counter -> base-unit number (None where unknown or duplicated)."""
    out: dict[tuple, dict] = {}
    for row in rows:
        counters = out.setdefault((row.get("id"), row.get("kernel")), {})
        metric = row.get("metric")
        counters[metric] = None if metric in counters else row.get("numeric_value")
    return out
