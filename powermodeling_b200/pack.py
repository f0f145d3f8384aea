"""Runner trial records -> the structure-of-arrays batch of ``pm_trials``.

Every field is extracted with the reference's coercion rules so the kernels
see exactly the values analysis.py would: ``_finite`` (analysis.py:70-77) maps
bools, non-numbers and non-finite numbers to None (NaN here); ``_samples``
(85-91) keeps the last sample of a duplicated timestamp and sorts by time;
``_throttle_mask`` (219-225) parses strings with base prefixes; epoch
boundaries fall back to nanosecond stamps (_measure_epochs, 245-251).
Record-level facts that need no telemetry arithmetic (process identity,
protocol fields, run quality) are folded into per-sample and per-trial flag
words; the per-trial issue strings they produce are returned to the caller.
"""
from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass, field

import numpy as np

from . import _native as N

TENSOR_WORKLOADS = {"tensor", "fp16_tensor", "tensor_fp16", "gemm"}
MEMORY_WORKLOADS = {"l1", "l2", "hbm"}
SFU_WORKLOADS = {"sfu_ex2", "sfu_lg2", "sfu_rcp", "sfu_rsqrt", "sfu_sqrt", "sfu_tanh"}
NONLINEAR_WORKLOADS = {"exp", "tanh", "silu", "rmsnorm", "softmax"}
ROW_WORKLOADS = {"rmsnorm", "softmax"}
PHASES = N.PHASE_NAMES
NAN = float("nan")


def finite(value) -> float | None:
    """The reference's _finite: float(value) when finite, else None."""
    kind = type(value)
    if kind is float:                      # the common cases first (bools are neither)
        return value if math.isfinite(value) else None
    if kind is int:
        return float(value)                # finite, or OverflowError as float() raises it
    if isinstance(value, bool):
        return None
    try:
        result = float(value)
    except (TypeError, ValueError):
        return None
    return result if math.isfinite(result) else None


def nan_if_none(value) -> float:
    if type(value) is float:               # the common case: no call into finite()
        return value if math.isfinite(value) else NAN
    v = finite(value)
    return NAN if v is None else v


def throttle_mask(value) -> int | None:
    try:
        if isinstance(value, str):
            return int(value, 0)
        return int(value) if value is not None else None
    except (ValueError, TypeError):
        return None


def workload_class(workload) -> int:
    if workload in TENSOR_WORKLOADS:
        return N.WL_TENSOR
    if workload in MEMORY_WORKLOADS:
        return N.WL_MEMORY
    if workload in SFU_WORKLOADS:
        return N.WL_SFU
    if workload in NONLINEAR_WORKLOADS:
        return N.WL_NONLINEAR
    return N.WL_OTHER


def phase_records(record: Mapping) -> dict:
    phases = record.get("phases", {})
    if isinstance(phases, list):
        phases = {p["name"]: p for p in phases if isinstance(p, dict) and "name" in p}
    return phases or {}


def sorted_samples(phase) -> list:
    """_samples: last observation wins on a duplicated timestamp; ascending time."""
    indexed = {}
    for item in (phase.get("samples", []) if isinstance(phase, Mapping) else []):
        if isinstance(item, dict) and (t := finite(item.get("t_s"))) is not None:
            indexed[t] = item
    return [indexed[t] for t in sorted(indexed)]


@dataclass
class Packed:
    """One batch: numpy arrays in pm_trials order plus host-side extras."""
    arrays: dict
    n_trials: int
    n_samples: int
    n_epochs: int
    max_phase_samples: int
    samples: list = field(default_factory=list)       # per slot: sorted sample dicts (for host-side lists)
    foreign_pids: list = field(default_factory=list)  # per slot: list of (index, pids)
    broadcast: int = 0                                # PM_COL_* bits of the one-element columns
    clock_repeat: bytes | bytearray | None = None    # per sample: 1 when its clocks read back as the previous sample's


class _Columns:
    def __init__(self):
        self.t, self.power, self.memory, self.gfx, self.sm, self.mem = [], [], [], [], [], []
        self.temp, self.plimit, self.enf, self.pstate = [], [], [], []
        self.e_int, self.e_float, self.throttle, self.flags, self.source = [], [], [], [], []


_SOURCE_IDS: dict = {}


def _source_id(source) -> int:
    if not source:
        return 0
    key = source if isinstance(source, str) else repr(source)
    if key not in _SOURCE_IDS:
        _SOURCE_IDS[key] = 1 + len(_SOURCE_IDS) % 15
    return _SOURCE_IDS[key]


def _pack_sample(s: dict, pid, cols: _Columns) -> list:
    cols.t.append(float(s["t_s"]))
    cols.power.append(nan_if_none(s.get("power_w")))
    cols.memory.append(nan_if_none(s.get("memory_power_w")))
    cols.gfx.append(nan_if_none(s.get("graphics_clock_mhz")))
    cols.sm.append(nan_if_none(s.get("sm_clock_mhz")))
    cols.mem.append(nan_if_none(s.get("memory_clock_mhz")))
    cols.temp.append(nan_if_none(s.get("temperature_c")))
    cols.plimit.append(nan_if_none(s.get("power_limit_w")))
    cols.enf.append(nan_if_none(s.get("enforced_power_limit_w")))
    cols.pstate.append(nan_if_none(s.get("pstate")))
    flags = 0
    counter = s.get("energy_mj")
    e_int, e_float = 0, NAN
    if type(counter) is int:
        flags |= N.S_ENERGY_ANCHOR
        e_int = counter
    if isinstance(counter, (int, float)) and not isinstance(counter, bool) and counter >= 0:
        if isinstance(counter, int):
            flags |= N.S_ENERGY_INT
            e_int = counter
        else:
            flags |= N.S_ENERGY_FLOAT
            e_float = float(counter)
    if e_int >= 1 << 63:
        e_int -= 1 << 64          # two's complement of a uint64 counter
    elif e_int < -(1 << 63):
        e_int = 0
    cols.e_int.append(e_int)
    cols.e_float.append(e_float)
    mask = throttle_mask(s.get("throttle_reasons"))
    if mask is not None and -(1 << 63) <= mask < (1 << 64):
        flags |= N.S_THROTTLE_VALID
        cols.throttle.append(mask - (1 << 64) if mask >= 1 << 63 else mask)
    else:
        cols.throttle.append(0)
    foreign = []
    for key, missing in (("compute_processes", N.S_NO_COMPUTE_INV), ("graphics_processes", N.S_NO_GRAPHICS_INV)):
        inventory = s.get(key)
        if not isinstance(inventory, list):
            flags |= missing
            continue
        if inventory and pid is None:
            flags |= N.S_PID_UNKNOWN
        for process in inventory:
            p = process.get("pid") if isinstance(process, dict) else process
            if p != pid:
                flags |= N.S_REF_FOREIGN
            if p is not None and p != pid:
                flags |= N.S_FOREIGN_PID
                foreign.append(p)
    if s.get("mps_compute_processes"):
        flags |= N.S_MPS
    if s.get("memory_power_w") is not None:
        flags |= N.S_MEMORY_POWER_SET
    cols.source.append(_source_id(s.get("memory_power_source")))
    cols.flags.append(flags)
    return foreign


def _epochs(bench: Mapping):
    """(status, list of epoch tuples) per the reference's parsing order."""
    source = bench.get("measure_epochs", bench.get("work_epochs"))
    if source is None:
        return N.EP_NONE, []
    if not isinstance(source, list) or not source:
        return N.EP_INVALID_LIST, []
    out = []
    for epoch in source:
        if not isinstance(epoch, dict):
            return N.EP_NON_DICT_AFTER, out
        a, b = finite(epoch.get("start_s")), finite(epoch.get("end_s"))
        if a is None:
            stamp = finite(epoch.get("host_monotonic_start_ns", epoch.get("start_ns")))
            a = stamp / 1e9 if stamp is not None else None
        if b is None:
            stamp = finite(epoch.get("host_monotonic_end_ns", epoch.get("end_ns")))
            b = stamp / 1e9 if stamp is not None else None
        out.append((NAN if a is None else a, NAN if b is None else b,
                    nan_if_none(epoch.get("operations")), nan_if_none(epoch.get("logical_bytes")),
                    nan_if_none(epoch.get("reference_loop_slots")), epoch.get("counts_exact") is True))
    return N.EP_OK, out


def _epoch_columns_python(arms: list):
    """(status per arm, epoch count per arm, the six epoch columns) by _epochs (the native parser's statement)."""
    status, counts, rows = [], [], []
    for source in arms:
        st, r = _epochs(source)
        status.append(st)
        counts.append(len(r))
        rows.extend(r)
    columns = tuple(np.asarray([r[k] for r in rows], dtype=np.float64) for k in range(5))
    columns += (np.asarray([r[5] for r in rows], dtype=np.uint8),)
    return np.asarray(status, dtype=np.int32), np.asarray(counts, dtype=np.int32), columns


def _epoch_columns_native(arms: list):
    status, counts, columns = _native_packer().epochs(arms, _epochs)
    cols = tuple(np.frombuffer(c, dtype=np.float64) for c in columns[:5]) + (np.frombuffer(columns[5], dtype=np.uint8),)
    return np.frombuffer(status, dtype=np.int32), np.frombuffer(counts, dtype=np.int32), cols


def tensor_flops_per_clock(record: Mapping, architectures: Mapping) -> float | None:
    """dense FLOP/SM/clock x SM count, or None when the reference's lookup would raise."""
    device = record.get("cuda_device") or record.get("device") or {}
    cc = device.get("compute_capability")
    try:
        if isinstance(cc, str):
            cc = tuple(int(x) for x in cc.split("."))
        elif isinstance(cc, (list, tuple)):
            cc = tuple(cc)
        else:
            cc = (device.get("cc_major", device.get("compute_capability_major")),
                  device.get("cc_minor", device.get("compute_capability_minor")))
        if cc not in architectures:
            return None
        value = architectures[cc]["dense_tensor_flops_per_sm_clock"] * device["sm_count"]
        return float(value * 1.0)
    except (ValueError, KeyError, TypeError):
        return None


SAMPLE_COLUMNS = (("t_s", np.float64), ("power_w", np.float64), ("memory_power_w", np.float64),
                  ("graphics_clock_mhz", np.float64), ("sm_clock_mhz", np.float64), ("memory_clock_mhz", np.float64),
                  ("temperature_c", np.float64), ("power_limit_w", np.float64), ("enforced_power_limit_w", np.float64),
                  ("pstate", np.float64), ("energy_int", np.int64), ("energy_float", np.float64),
                  ("throttle_reasons", np.int64), ("sample_flags", np.uint16), ("memory_power_source", np.uint8))


def _native_packer():
    try:
        from . import _packnative
    except ImportError as exc:
        raise N.NativeError("the record packer extension (_packnative) is not built; run powermodeling_b200.build") from exc
    return _packnative


def _pack_slots_python(slot_raw: list, slot_pid: list):
    """The per-sample packing in Python (the native packer's specification; tests compare the two)."""
    cols = _Columns()
    counts, slot_samples, slot_foreign = [], [], []
    for raw, pid in zip(slot_raw, slot_pid):
        samples = sorted_samples({"samples": raw})
        foreign = []
        for i, s in enumerate(samples):
            f = _pack_sample(s, pid, cols)
            if f:
                foreign.append((i, f))
        counts.append(len(samples))
        slot_samples.append(samples)
        slot_foreign.append(foreign)
    lists = (cols.t, cols.power, cols.memory, cols.gfx, cols.sm, cols.mem, cols.temp, cols.plimit, cols.enf,
             cols.pstate, cols.e_int, cols.e_float, cols.throttle, cols.flags, cols.source)
    arrays = {name: np.asarray(values, dtype=dtype) for (name, dtype), values in zip(SAMPLE_COLUMNS, lists)}
    return arrays, counts, slot_samples, slot_foreign


def _pack_slots_native(slot_raw: list, slot_pid: list):
    columns, counts, slot_samples, slot_foreign = _native_packer().pack(slot_raw, slot_pid, _SOURCE_IDS)
    # views of the bytearrays the packer filled (no copy)
    arrays = {name: np.frombuffer(columns[name], dtype=dtype) for name, dtype in SAMPLE_COLUMNS}
    arrays["clock_repeat"] = columns["clock_repeat"]
    return arrays, counts, slot_samples, slot_foreign


def pack_trials(records: list, host_flags: list, architectures: Mapping, native: bool = True) -> Packed:
    """Build the pm_trials arrays for ``records``; ``host_flags[i]`` are extra trial flag bits.

    The per-sample work (sorting, coercion, flags) runs in the native packer;
    ``native=False`` runs the same rules in Python."""
    nt = len(records)
    offsets = np.zeros(nt * N.PM_PHASES + 1, dtype=np.int64)
    starts = np.full(nt * N.PM_PHASES, NAN)
    ends = np.full(nt * N.PM_PHASES, NAN)
    present = np.zeros(nt * N.PM_PHASES, dtype=np.uint8)
    ep_off = np.zeros(nt * 2 + 1, dtype=np.int32)
    ep_status = np.zeros(nt * 2, dtype=np.int32)
    scalars = np.full((nt, N.TS_COUNT), NAN)
    tflags = np.zeros(nt, dtype=np.uint32)
    slot_raw, slot_pid = [], []
    arms = []                                        # per (trial, arm): the mapping holding its epoch list
    for t, record in enumerate(records):
        phases = phase_records(record)
        pid = (record.get("quality") or {}).get("measurement_pid")
        for p, name in enumerate(PHASES):
            slot = t * N.PM_PHASES + p
            phase = phases.get(name)
            raw = []
            if phase and (type(phase) is dict or isinstance(phase, Mapping)):
                present[slot] = 1
                starts[slot] = nan_if_none(phase.get("start_s"))
                ends[slot] = nan_if_none(phase.get("end_s"))
                raw = phase.get("samples", [])
            slot_raw.append(raw)
            slot_pid.append(pid)
        bench = record.get("benchmark") or record.get("result") or {}
        reference = record.get("active_reference") or {}
        arms.append(bench)
        arms.append(reference)
        config = dict(record.get("config") or {})
        device = record.get("device") or {}
        sc = scalars[t]
        sc[N.TS["BENCH_DURATION_S"]] = nan_if_none(bench.get("duration_s"))
        sc[N.TS["BENCH_HOST_DURATION_S"]] = nan_if_none(bench.get("host_duration_s"))
        sc[N.TS["BENCH_OPERATIONS"]] = nan_if_none(bench.get("operations"))
        sc[N.TS["BENCH_LOGICAL_BYTES"]] = nan_if_none(bench.get("logical_bytes"))
        sc[N.TS["REF_OPERATIONS"]] = nan_if_none(reference.get("operations"))
        sc[N.TS["REF_LOGICAL_BYTES"]] = nan_if_none(reference.get("logical_bytes"))
        sc[N.TS["REQ_GRAPHICS_MHZ"]] = nan_if_none(config.get("graphics_clock_mhz"))
        sc[N.TS["REQ_MEMORY_MHZ"]] = nan_if_none(config.get("memory_clock_mhz"))
        sc[N.TS["REQ_SM_MHZ"]] = nan_if_none(config.get("sm_clock_mhz"))
        fallback = (finite(record.get("power_limit_w", device.get("power_limit_w", config.get("power_limit_w"))))
                    or finite((device.get("sample") or {}).get("power_limit_w")))
        sc[N.TS["POWER_LIMIT_FALLBACK_W"]] = NAN if fallback is None else fallback
        workload = record.get("workload")
        flags = workload_class(workload) | host_flags[t]
        if workload in TENSOR_WORKLOADS:
            fpc = tensor_flops_per_clock(record, architectures)
            if fpc is not None:
                sc[N.TS["TENSOR_FLOPS_PER_CLOCK"]] = fpc
                flags |= N.T_TENSOR_PEAK_KNOWN
        if workload in ROW_WORKLOADS:
            flags |= N.T_ROWWISE
            sc[N.TS["ROW_WIDTH"]] = nan_if_none(bench.get("row_width"))
        protocol = record.get("treatment_protocol") or bench.get("treatment_protocol") or {}
        if protocol.get("order") == "AB":
            flags |= N.T_ORDER_AB
        elif protocol.get("order") == "BA":
            flags |= N.T_ORDER_BA
        tflags[t] = flags
    epochs = _epoch_columns_native(arms) if native else _epoch_columns_python(arms)
    ep_status[:] = epochs[0]
    np.cumsum(epochs[1], out=ep_off[1:])
    sample_arrays, counts, slot_samples, slot_foreign = (_pack_slots_native if native else _pack_slots_python)(slot_raw, slot_pid)
    clock_repeat = sample_arrays.pop("clock_repeat", None)   # host only (the Python packer leaves it out)
    np.cumsum(counts, out=offsets[1:])
    ns = int(offsets[-1])
    longest = max(counts, default=0)
    arrays = {
        "phase_offsets": offsets, "phase_start_s": starts, "phase_end_s": ends, "phase_present": present,
        **sample_arrays,
        "epoch_offsets": ep_off, "epoch_status": ep_status,
        "epoch_start_s": epochs[2][0], "epoch_end_s": epochs[2][1], "epoch_operations": epochs[2][2],
        "epoch_logical_bytes": epochs[2][3], "epoch_loop_slots": epochs[2][4], "epoch_counts_exact": epochs[2][5],
        "trial_scalars": np.ascontiguousarray(scalars.reshape(-1)), "trial_flags": tflags,
    }
    broadcast = broadcast_constant_columns(arrays, ns)
    return Packed(arrays, nt, ns, int(ep_off[-1]), longest, slot_samples, slot_foreign, broadcast, clock_repeat)


def broadcast_constant_columns(arrays: dict, n_samples: int) -> int:
    """Replace every per-sample column whose samples are bitwise identical by its first element.

    Returns the PM_COL_* bits of the replaced columns.  Bitwise comparison
    keeps NaN payloads and signed zeros exactly as the samples had them, so
    the kernel reads the same value for every sample either way.
    """
    bits = 0
    if n_samples == 0:
        return 0
    ints = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}
    for name, bit in N.BROADCAST_COLUMNS:
        a = arrays[name]
        raw = a.view(ints[a.itemsize])
        if (raw == raw[0]).all():
            arrays[name] = np.ascontiguousarray(a[:1])
            bits |= bit
    return bits


def trials_struct(p: Packed) -> N.Trials:
    """A pm_trials view of packed host arrays (the arrays must outlive it)."""
    t = N.Trials()
    t.n_trials, t.max_phase_samples, t.n_samples, t.n_epochs = p.n_trials, p.max_phase_samples, p.n_samples, p.n_epochs
    for name, dtype, _ in N.TRIAL_ARRAYS + N.EPOCH_ARRAYS + N.TAIL_ARRAYS:
        a = p.arrays[name]
        assert a.dtype == dtype and a.flags["C_CONTIGUOUS"], name
        setattr(t, name, a.ctypes.data if a.size else None)
    t.broadcast_columns = p.broadcast
    return t
