"""NVML telemetry backed by the native sampler in libpmb200.so.

Same surface as powermodeling/telemetry.py: ``NvmlDevice(index, uuid,
nvml_module)`` with ``read_sample``/``sample``/``metadata``/``close`` and
``capabilities``; ``Sampler(device, interval_s)`` with ``start``/``stop``/
``samples``/``error``; ``TelemetryError``.  A sample is the reference's
dictionary (telemetry.py:195-243) built from the fixed ``pm_nvml_sample``
struct the native code fills.

The reads themselves, their checks, their timestamps and the sampling thread
are native (pm_nvml_*, pm_sampler_*).  ``nvml_module=None`` reads
libnvidia-ml.so.1 directly; any other object with the pynvml call surface is
wrapped into the native backend table (``_ModuleBackend``), which is how the
hardware-free tests inject a fake driver — the counterpart of the reference's
``nvml_module`` hook (telemetry.py:58-65).
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Any

from ._native import library

# --------------------------------------------------------------------------- ABI
PM_OK, PM_E_INVALID, PM_E_NVML, PM_E_TIMEOUT, PM_E_STATE = 0, -1, -5, -6, -7
TE_VALUE, TE_FIELD_COUNT, TE_FIELD_ID, TE_FIELD_SCOPE = 0x10001, 0x10002, 0x10003, 0x10004
TE_VALUE_TYPE, TE_LOCK, TE_PID, TE_CLOSED = 0x10005, 0x10006, 0x10007, 0x10008
TE_FOREIGN_BASE = 0x1000000
TS_ENERGY_DECREASED, TS_FATAL, TS_FIELDS_QUERIED = 1, 2, 4
N_FIELDS = 19
(TF_POWER, TF_POWER_INSTANT, TF_POWER_AVERAGE, TF_MEMORY_INSTANT, TF_MEMORY_AVERAGE, TF_ENERGY, TF_GRAPHICS_CLOCK,
 TF_SM_CLOCK, TF_MEMORY_CLOCK, TF_TEMPERATURE, TF_PSTATE, TF_THROTTLE, TF_UTILIZATION, TF_POWER_LIMIT,
 TF_ENFORCED_LIMIT, TF_COMPUTE_PROCS, TF_GRAPHICS_PROCS, TF_MPS_PROCS, TF_FIELD_QUERY) = range(N_FIELDS)
UINT64_MAX = (1 << 64) - 1


class _Value(C.Union):
    _fields_ = [("d", C.c_double), ("ui", C.c_uint32), ("ul", C.c_uint64), ("ull", C.c_uint64), ("sll", C.c_int64)]


class Field(C.Structure):
    _fields_ = [("field_id", C.c_uint32), ("scope_id", C.c_uint32), ("timestamp_us", C.c_int64),
                ("latency_us", C.c_int64), ("value_type", C.c_int32), ("ret", C.c_int32),
                ("value_error", C.c_int32), ("meta_error", C.c_int32), ("value", _Value)]


class Process(C.Structure):
    _fields_ = [("pid", C.c_uint64), ("used_bytes", C.c_uint64)]


_vp = C.c_void_p
_F_INIT = C.CFUNCTYPE(C.c_int, _vp)
_F_BY_UUID = C.CFUNCTYPE(C.c_int, _vp, C.c_char_p, C.POINTER(_vp))
_F_BY_INDEX = C.CFUNCTYPE(C.c_int, _vp, C.c_uint32, C.POINTER(_vp))
_F_UUID = C.CFUNCTYPE(C.c_int, _vp, _vp, C.c_void_p, C.c_uint32)
_F_DOUBLE = C.CFUNCTYPE(C.c_int, _vp, _vp, C.POINTER(C.c_double))
_F_FIELDS = C.CFUNCTYPE(C.c_int, _vp, _vp, C.c_int, C.POINTER(Field))
_F_U64 = C.CFUNCTYPE(C.c_int, _vp, _vp, C.POINTER(C.c_uint64))
_F_CLOCK = C.CFUNCTYPE(C.c_int, _vp, _vp, C.c_int, C.POINTER(C.c_uint64))
_F_I64 = C.CFUNCTYPE(C.c_int, _vp, _vp, C.POINTER(C.c_int64))
_F_UTIL = C.CFUNCTYPE(C.c_int, _vp, _vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64))
_F_PROCS = C.CFUNCTYPE(C.c_int, _vp, _vp, C.c_int, C.POINTER(C.c_uint32), C.POINTER(Process))
_F_FATAL = C.CFUNCTYPE(C.c_int, _vp, C.c_int)


class Backend(C.Structure):
    _fields_ = [("ctx", _vp), ("init", _F_INIT), ("shutdown", _F_INIT), ("handle_by_uuid", _F_BY_UUID),
                ("handle_by_index", _F_BY_INDEX), ("uuid", _F_UUID), ("power_usage", _F_DOUBLE),
                ("field_values", _F_FIELDS), ("total_energy", _F_U64), ("clock", _F_CLOCK),
                ("temperature", _F_I64), ("pstate", _F_I64), ("throttle_reasons", _F_U64),
                ("utilization", _F_UTIL), ("power_limit", _F_DOUBLE), ("enforced_power_limit", _F_DOUBLE),
                ("processes", _F_PROCS), ("is_fatal", _F_FATAL), ("field_id", C.c_uint32 * 4),
                ("scope_id", C.c_uint32 * 4), ("field_missing", C.c_int32 * 4)]


class Sample(C.Structure):
    _fields_ = [("t_s", C.c_double), ("query_start_s", C.c_double), ("query_end_s", C.c_double),
                ("query_duration_s", C.c_double), ("query_realtime_start_s", C.c_double),
                ("query_realtime_end_s", C.c_double), ("power_mw", C.c_double), ("field_mw", C.c_double * 4),
                ("field_timestamp_us", C.c_int64 * 4), ("field_latency_us", C.c_int64 * 4),
                ("energy_mj", C.c_uint64), ("graphics_clock_mhz", C.c_uint64), ("sm_clock_mhz", C.c_uint64),
                ("memory_clock_mhz", C.c_uint64), ("temperature_c", C.c_int64), ("pstate", C.c_int64),
                ("throttle_reasons", C.c_uint64), ("gpu_utilization_percent", C.c_int64),
                ("memory_utilization_percent", C.c_int64), ("power_limit_mw", C.c_double),
                ("enforced_power_limit_mw", C.c_double), ("process_offset", C.c_uint32 * 3),
                ("process_count", C.c_uint32 * 3), ("code", C.c_int32 * N_FIELDS),
                ("field_value_type", C.c_int32 * 4), ("flags", C.c_uint32), ("sequence", C.c_uint32)]


class Metadata(C.Structure):
    _fields_ = [("name", C.c_char * 96), ("pci_bus_id", C.c_char * 32), ("driver_version", C.c_char * 80),
                ("nvml_version", C.c_char * 80), ("cc_major", C.c_int64), ("cc_minor", C.c_int64),
                ("memory_total", C.c_uint64), ("memory_used", C.c_uint64), ("memory_free", C.c_uint64),
                ("mig_current", C.c_int64), ("mig_pending", C.c_int64), ("persistence_mode", C.c_int64),
                ("ecc_current", C.c_int64), ("ecc_pending", C.c_int64), ("power_limit_min_mw", C.c_double),
                ("power_limit_max_mw", C.c_double), ("default_power_limit_mw", C.c_double),
                ("code", C.c_int32 * 11)]


def _lib():
    lib = library()
    if getattr(lib, "_pm_telemetry_bound", False):
        return lib
    P = C.POINTER
    sig = {
        "pm_nvml_open": (C.c_int, [P(Backend), C.c_uint32, C.c_char_p, P(_vp)]),
        "pm_nvml_close": (C.c_int, [_vp]),
        "pm_nvml_uuid": (C.c_int, [_vp, C.c_char_p, C.c_size_t]),
        "pm_nvml_read_sample": (C.c_int, [_vp, P(Sample), P(Process), C.c_uint32]),
        "pm_nvml_read_metadata": (C.c_int, [_vp, P(Metadata)]),
        "pm_nvml_active_samplers": (C.c_int, [_vp]),
        "pm_nvml_error_string": (C.c_char_p, [C.c_int]),
        "pm_sampler_create": (C.c_int, [_vp, C.c_double, P(_vp)]),
        "pm_sampler_start": (C.c_int, [_vp, C.c_double]),
        "pm_sampler_stop": (C.c_int, [_vp, C.c_double]),
        "pm_sampler_count": (C.c_int, [_vp, P(C.c_uint64), P(C.c_uint64)]),
        "pm_sampler_copy": (C.c_int, [_vp, C.c_uint64, C.c_uint64, P(Sample), P(Process), C.c_uint64]),
        "pm_sampler_status": (C.c_int, [_vp, P(C.c_int), P(C.c_uint64), P(C.c_int)]),
        "pm_sampler_destroy": (C.c_int, [_vp]),
        "pm_clock_watch_start": (C.c_int, [_vp, C.c_double, P(_vp)]),
        "pm_clock_watch_stop": (C.c_int, [_vp, _vp, _vp, _vp, _vp, C.c_uint64, P(C.c_uint64)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    lib._pm_telemetry_bound = True
    return lib


def _last_error() -> str:
    lib = library()
    buf = C.create_string_buffer(1024)
    lib.pm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


# --------------------------------------------------------------------------- reference helpers
class TelemetryError(RuntimeError):
    """An operation needed to identify or monitor the selected GPU failed."""


def _error(exc: BaseException) -> dict[str, Any]:
    """Error record of one failed read (telemetry.py:25-29)."""
    result = {"type": type(exc).__name__, "message": str(exc)}
    if getattr(exc, "value", None) is not None:
        result["code"] = int(exc.value)
    return result


def _text(value: Any) -> str:
    return value.decode("utf-8", errors="replace") if isinstance(value, bytes) else str(value)


def _number(value: Any) -> float:
    """Nonnegative finite number (telemetry.py:36-40)."""
    result = float(value)
    if not math.isfinite(result) or result < 0:
        raise ValueError(f"Invalid nonnegative telemetry value: {value!r}")
    return result


def _integer(value: Any) -> int:
    """Nonnegative integer, without a float round trip (telemetry.py:43-48)."""
    result = int(value)
    if isinstance(value, bool) or result < 0 or result != value:
        raise ValueError(f"Invalid nonnegative integer telemetry value: {value!r}")
    return result


# NVML return codes -> the error class names pynvml derives from them.
_NVML_ERROR_NAMES = {
    1: "Uninitialized", 2: "InvalidArgument", 3: "NotSupported", 4: "NoPermission", 5: "AlreadyInitialized",
    6: "NotFound", 7: "InsufficientSize", 8: "InsufficientPower", 9: "DriverNotLoaded", 10: "Timeout",
    11: "IrqIssue", 12: "LibraryNotFound", 13: "FunctionNotFound", 14: "CorruptedInforom", 15: "GpuIsLost",
    16: "ResetRequired", 17: "OperatingSystem", 18: "LibRmVersionMismatch", 19: "InUse", 20: "Memory",
    21: "NoData", 22: "VgpuEccNotSupported", 23: "InsufficientResources", 24: "FreqNotSupported",
    25: "ArgumentVersionMismatch", 26: "Deprecated", 27: "NotReady", 28: "GpuNotFound", 29: "InvalidState",
    999: "Unknown",
}
_FATAL_DEFAULTS = (("NVML_ERROR_UNINITIALIZED", 1), ("NVML_ERROR_GPU_IS_LOST", 15),
                   ("NVML_ERROR_RESET_REQUIRED", 16), ("NVML_ERROR_LIB_RM_VERSION_MISMATCH", 18))
# Clock event reason bits in the order pynvml's sorted constant names give
# (telemetry.py:257-267 reads them from the module; the native backend has no module).
_THROTTLE_BITS = (("ApplicationsClocksSetting", 0x2), ("DisplayClockSetting", 0x100), ("GpuIdle", 0x1),
                  ("HwPowerBrakeSlowdown", 0x80), ("HwSlowdown", 0x8), ("HwThermalSlowdown", 0x40),
                  ("SwPowerCap", 0x4), ("SwThermalSlowdown", 0x20), ("SyncBoost", 0x10))

_POWER_SPECS = (("power_instant_w", "NVML_FI_DEV_POWER_INSTANT", "NVML_POWER_SCOPE_GPU", "gpu"),
                ("power_average_w", "NVML_FI_DEV_POWER_AVERAGE", "NVML_POWER_SCOPE_GPU", "gpu"),
                ("memory_power_instant_w", "NVML_FI_DEV_POWER_INSTANT", "NVML_POWER_SCOPE_MEMORY", "memory"),
                ("memory_power_average_w", "NVML_FI_DEV_POWER_AVERAGE", "NVML_POWER_SCOPE_MEMORY", "memory"))
_NATIVE_FIELD_IDS = {"NVML_FI_DEV_POWER_INSTANT": 186, "NVML_FI_DEV_POWER_AVERAGE": 185}
_NATIVE_SCOPES = {"NVML_POWER_SCOPE_GPU": 0, "NVML_POWER_SCOPE_MEMORY": 2}
_PROCESS_APIS = ("nvmlDeviceGetComputeRunningProcesses", "nvmlDeviceGetGraphicsRunningProcesses",
                 "nvmlDeviceGetMPSComputeRunningProcesses")
_PROCESS_KEYS = ("compute_processes", "graphics_processes", "mps_compute_processes")


# --------------------------------------------------------------------------- module backend
class _ModuleBackend:
    """Wraps a pynvml-like module into the native backend table.

    Each slot calls the module function the reference calls and applies the
    reference's transform (``_number``, ``_integer``, ``int``) before the value
    crosses into C; an exception becomes a foreign code whose error record
    (``_error``) the sample converter looks up again.
    """

    def __init__(self, module: Any):
        self.nvml = module
        self._records: list[dict] = []
        self._interned: dict[tuple, int] = {}
        self.last_exception: BaseException | None = None
        self._handles: list[Any] = []
        self.fatal_codes = {getattr(module, name, default) for name, default in _FATAL_DEFAULTS}
        self.throttle_api = ("nvmlDeviceGetCurrentClocksEventReasons"
                             if hasattr(module, "nvmlDeviceGetCurrentClocksEventReasons")
                             else "nvmlDeviceGetCurrentClocksThrottleReasons")
        t = Backend()
        # One backend context per module object: devices on the same module
        # share one nvmlInit/nvmlShutdown session (telemetry.py:66-71, 318-326).
        t.ctx = id(module)
        keep = []

        def slot(ftype, fn):
            cb = ftype(fn)
            keep.append(cb)
            return cb

        t.init = slot(_F_INIT, lambda ctx: self._call(lambda: module.nvmlInit()))
        t.shutdown = slot(_F_INIT, lambda ctx: self._call(lambda: module.nvmlShutdown()))
        t.handle_by_uuid = slot(_F_BY_UUID, self._by_uuid)
        t.handle_by_index = slot(_F_BY_INDEX, self._by_index)
        t.uuid = slot(_F_UUID, self._uuid)
        t.power_usage = slot(_F_DOUBLE, lambda c, h, out: self._scalar(out, "nvmlDeviceGetPowerUsage", h, _number))
        t.field_values = slot(_F_FIELDS, self._fields)
        t.total_energy = slot(_F_U64, lambda c, h, out: self._scalar(out, "nvmlDeviceGetTotalEnergyConsumption", h,
                                                                   _integer))
        t.clock = slot(_F_CLOCK, self._clock)
        t.temperature = slot(_F_I64, lambda c, h, out: self._scalar(
            out, "nvmlDeviceGetTemperature", h, int, getattr(module, "NVML_TEMPERATURE_GPU", 0)))
        t.pstate = slot(_F_I64, lambda c, h, out: self._scalar(out, "nvmlDeviceGetPerformanceState", h, int))
        t.throttle_reasons = slot(_F_U64, lambda c, h, out: self._scalar(out, self.throttle_api, h, int))
        t.utilization = slot(_F_UTIL, self._utilization)
        t.power_limit = slot(_F_DOUBLE, lambda c, h, out: self._scalar(out, "nvmlDeviceGetPowerManagementLimit", h,
                                                                     _number))
        t.enforced_power_limit = slot(_F_DOUBLE, lambda c, h, out: self._scalar(
            out, "nvmlDeviceGetEnforcedPowerLimit", h, _number))
        t.processes = slot(_F_PROCS, self._processes)
        t.is_fatal = slot(_F_FATAL, self._is_fatal)
        for i, (key, field_name, scope_name, _) in enumerate(_POWER_SPECS):
            try:
                # Missing scope constants cannot be replaced with guessed IDs.
                t.field_id[i] = int(getattr(module, field_name))
                t.scope_id[i] = int(getattr(module, scope_name))
                t.field_missing[i] = 0
            except AttributeError as exc:
                t.field_missing[i] = self._foreign(exc)
        self.table = t
        self._keep = keep

    # -- error records
    def _foreign(self, exc: BaseException) -> int:
        self.last_exception = exc
        record = _error(exc)
        key = (record["type"], record["message"], record.get("code"))
        code = self._interned.get(key)
        if code is None:
            code = TE_FOREIGN_BASE + len(self._records)
            self._records.append(record)
            self._interned[key] = code
        return code

    def record(self, code: int) -> dict:
        return dict(self._records[code - TE_FOREIGN_BASE])

    def _call(self, fn) -> int:
        try:
            fn()
            return 0
        except BaseException as exc:  # noqa: BLE001 - every failure is a recorded field error
            return self._foreign(exc)

    def _is_fatal(self, ctx, code: int) -> int:
        if code >= TE_FOREIGN_BASE:
            return int(self._records[code - TE_FOREIGN_BASE].get("code") in self.fatal_codes)
        # A raw NVML code of a power field carries its code only when the
        # module has an NVMLError class to raise (telemetry.py:150-155).
        return int(getattr(self.nvml, "NVMLError", None) is not None and code in self.fatal_codes)

    def _handle(self, token) -> Any:
        return self._handles[int(token or 0) - 1]

    def _by_uuid(self, ctx, uuid, out):
        def run():
            self._handles.append(self.nvml.nvmlDeviceGetHandleByUUID(uuid.decode()))
            out[0] = len(self._handles)
        return self._call(run)

    def _by_index(self, ctx, index, out):
        def run():
            self._handles.append(self.nvml.nvmlDeviceGetHandleByIndex(int(index)))
            out[0] = len(self._handles)
        return self._call(run)

    def _uuid(self, ctx, h, buf, size):
        def run():
            text = _text(self.nvml.nvmlDeviceGetUUID(self._handle(h))).encode()[: max(0, size - 1)]
            C.memmove(buf, text + b"\0", len(text) + 1)
        return self._call(run)

    def _scalar(self, out, api, h, transform, *args):
        def run():
            out[0] = transform(getattr(self.nvml, api)(self._handle(h), *args))
        return self._call(run)

    def _clock(self, ctx, h, kind, out):
        names = (("NVML_CLOCK_GRAPHICS", 0), ("NVML_CLOCK_SM", 1), ("NVML_CLOCK_MEM", 2))
        name, default = names[kind]
        return self._scalar(out, "nvmlDeviceGetClockInfo", h, _integer, getattr(self.nvml, name, default))

    def _utilization(self, ctx, h, gpu, mem):
        def run():
            v = self.nvml.nvmlDeviceGetUtilizationRates(self._handle(h))
            g, m = int(v.gpu), int(v.memory)
            gpu[0], mem[0] = g, m
        return self._call(run)

    def _processes(self, ctx, h, kind, count, out):
        try:
            unavailable = getattr(self.nvml, "NVML_VALUE_NOT_AVAILABLE", UINT64_MAX)
            items = []
            for process in getattr(self.nvml, _PROCESS_APIS[kind])(self._handle(h)):
                used = getattr(process, "usedGpuMemory", None)
                pid = _integer(process.pid)
                if pid == 0:
                    raise ValueError("NVML process inventory must contain positive process IDs")
                items.append((pid, UINT64_MAX if used in (None, unavailable) else _integer(used)))
        except BaseException as exc:  # noqa: BLE001
            return self._foreign(exc)
        if len(items) > count[0]:
            count[0] = len(items)
            return 7  # NVML_ERROR_INSUFFICIENT_SIZE: the caller retries with room for all
        for i, (pid, used) in enumerate(items):
            out[i].pid, out[i].used_bytes = pid, used
        count[0] = len(items)
        return 0

    def _fields(self, ctx, h, count, fields):
        try:
            request = [(fields[i].field_id, fields[i].scope_id) for i in range(count)]
            values = self.nvml.nvmlDeviceGetFieldValues(self._handle(h), request)
            if len(values) != count:
                return TE_FIELD_COUNT
        except BaseException as exc:  # noqa: BLE001
            return self._foreign(exc)
        types = {getattr(self.nvml, "NVML_VALUE_TYPE_DOUBLE", 0): "dVal",
                 getattr(self.nvml, "NVML_VALUE_TYPE_UNSIGNED_INT", 1): "uiVal",
                 getattr(self.nvml, "NVML_VALUE_TYPE_UNSIGNED_LONG", 2): "ulVal",
                 getattr(self.nvml, "NVML_VALUE_TYPE_UNSIGNED_LONG_LONG", 3): "ullVal",
                 getattr(self.nvml, "NVML_VALUE_TYPE_SIGNED_LONG_LONG", 4): "sllVal"}
        for i, field in enumerate(values):
            f = fields[i]
            f.value_error = f.meta_error = 0
            try:
                f.ret = int(field.nvmlReturn)
            except BaseException as exc:  # noqa: BLE001
                f.ret = self._foreign(exc)
                continue
            try:
                if hasattr(field, "fieldId"):
                    f.field_id = int(field.fieldId)
                if hasattr(field, "scopeId"):
                    f.scope_id = int(field.scopeId)
                value_type = int(field.valueType)
            except BaseException as exc:  # noqa: BLE001
                f.ret = self._foreign(exc)
                continue
            member = types.get(value_type)
            if member is None:
                # Unsupported: the native check rejects any type outside 0..4.
                f.value_type = value_type if not 0 <= value_type <= 4 else -1
                continue
            # Values cross as doubles: the reference converts them with float().
            f.value_type = 0
            try:
                f.value.d = _number(getattr(field.value, member))
            except BaseException as exc:  # noqa: BLE001
                f.value_error = self._foreign(exc)
                continue
            try:
                f.timestamp_us = int(field.timestamp)
                f.latency_us = int(field.latencyUsec)
            except BaseException as exc:  # noqa: BLE001
                f.meta_error = self._foreign(exc)
        return 0


# --------------------------------------------------------------------------- sample conversion
class _Converter:
    """Builds the reference's sample dictionary from a native sample."""

    def __init__(self, device: "NvmlDevice"):
        self.device = device
        self.backend = device._backend
        self.nvml = device.nvml

    def error(self, code: int, *, field: bool = False, raw: Any = None) -> dict:
        if code >= TE_FOREIGN_BASE:
            return self.backend.record(code)
        if code == TE_VALUE:
            return {"type": "ValueError", "message": f"Invalid nonnegative telemetry value: {raw!r}"}
        if code == TE_FIELD_COUNT:
            return {"type": "TelemetryError", "message": "NVML field query returned the wrong number of values"}
        if code == TE_FIELD_ID:
            return {"type": "TelemetryError", "message": "NVML returned a field with the wrong field ID"}
        if code == TE_FIELD_SCOPE:
            return {"type": "TelemetryError", "message": "NVML returned a field with the wrong power scope"}
        if code == TE_VALUE_TYPE:
            return {"type": "TelemetryError", "message": f"Unsupported NVML value type {raw}"}
        if code == TE_PID:
            return {"type": "ValueError", "message": "NVML process inventory must contain positive process IDs"}
        if code in (TE_LOCK, TE_CLOSED):
            return {"type": "TelemetryError", "message": "Another NVML query is still running; refusing concurrent "
                    "driver access" if code == TE_LOCK else "NVML device is closed"}
        if self.backend is not None:
            error_class = getattr(self.nvml, "NVMLError", None)
            if error_class is not None:
                return _error(error_class(code))
            return {"type": "TelemetryError", "message": f"NVML field returned error code {code}"}
        message = _lib().pm_nvml_error_string(code)
        name = _NVML_ERROR_NAMES.get(code)
        return {"type": f"NVMLError_{name}" if name else "NVMLError",
                "message": message.decode() if message else f"NVML error {code}", "code": code}

    def fatal_codes(self) -> set:
        if self.backend is not None:
            return self.backend.fatal_codes
        return {code for _, code in _FATAL_DEFAULTS}

    def throttle_names(self, value: int) -> list[str]:
        if self.backend is None:
            return [name for name, bit in _THROTTLE_BITS if value & bit]
        names, seen = [], set()
        for prefix in ("nvmlClocksEventReason", "nvmlClocksThrottleReason"):
            for name in sorted(dir(self.nvml)):
                if name.startswith(prefix) and not name.endswith(("All", "None")):
                    bit = getattr(self.nvml, name)
                    if isinstance(bit, int) and bit > 0 and bit & (bit - 1) == 0 and value & bit and bit not in seen:
                        names.append(name[len(prefix):])
                        seen.add(bit)
        return names

    def throttle_api(self) -> str:
        if self.backend is not None:
            return self.backend.throttle_api
        return "nvmlDeviceGetCurrentClocksEventReasons"

    def convert(self, s: Sample, procs) -> dict[str, Any]:
        caps = self.device.capabilities
        r: dict[str, Any] = {"uuid": self.device.uuid, "errors": {}, "field_metadata": {}}
        code = s.code

        def put(key, api, slot, value, raw=None):
            if code[slot]:
                r[key] = None
                err = self.error(code[slot], raw=raw)
                r["errors"][key] = err
                caps[key] = {"available": False, "api": api, "error": err}
                return None
            r[key] = value
            caps[key] = {"available": True, "api": api}
            return value

        put("power_w", "nvmlDeviceGetPowerUsage", TF_POWER, s.power_mw / 1000, raw=s.power_mw)
        self._power_fields(r, s, caps)
        energy = put("energy_mj", "nvmlDeviceGetTotalEnergyConsumption", TF_ENERGY, int(s.energy_mj))
        r["energy_counter_decreased"] = False
        if energy is not None and s.flags & TS_ENERGY_DECREASED:
            r["energy_counter_decreased"] = True
            r["errors"]["energy_counter"] = {"type": "CounterDecrease", "message": "Energy counter decreased: driver "
                                             "reset or counter rollover; do not subtract across this boundary"}
        put("graphics_clock_mhz", "nvmlDeviceGetClockInfo", TF_GRAPHICS_CLOCK, int(s.graphics_clock_mhz))
        put("sm_clock_mhz", "nvmlDeviceGetClockInfo", TF_SM_CLOCK, int(s.sm_clock_mhz))
        put("memory_clock_mhz", "nvmlDeviceGetClockInfo", TF_MEMORY_CLOCK, int(s.memory_clock_mhz))
        put("temperature_c", "nvmlDeviceGetTemperature", TF_TEMPERATURE, int(s.temperature_c))
        put("pstate", "nvmlDeviceGetPerformanceState", TF_PSTATE, int(s.pstate))
        throttle = put("throttle_reasons", self.throttle_api(), TF_THROTTLE, int(s.throttle_reasons))
        r["throttle_reason_names"] = self.throttle_names(throttle) if throttle is not None else None
        util = put("utilization", "nvmlDeviceGetUtilizationRates", TF_UTILIZATION,
                   {"gpu_percent": int(s.gpu_utilization_percent),
                    "memory_percent": int(s.memory_utilization_percent)})
        r["gpu_utilization_percent"] = util["gpu_percent"] if util else None
        r["memory_utilization_percent"] = util["memory_percent"] if util else None
        put("power_limit_w", "nvmlDeviceGetPowerManagementLimit", TF_POWER_LIMIT, s.power_limit_mw / 1000,
            raw=s.power_limit_mw)
        put("enforced_power_limit_w", "nvmlDeviceGetEnforcedPowerLimit", TF_ENFORCED_LIMIT,
            s.enforced_power_limit_mw / 1000, raw=s.enforced_power_limit_mw)
        for kind, (key, api) in enumerate(zip(_PROCESS_KEYS, _PROCESS_APIS)):
            base, n = s.process_offset[kind], s.process_count[kind]
            items = [{"pid": int(procs[base + i].pid),
                      "used_gpu_memory_bytes": None if procs[base + i].used_bytes == UINT64_MAX
                      else int(procs[base + i].used_bytes)} for i in range(n)]
            put(key, api, TF_COMPUTE_PROCS + kind, items)
        r.update(t_s=s.t_s, query_start_s=s.query_start_s, query_end_s=s.query_end_s,
                 query_duration_s=s.query_duration_s, query_realtime_start_s=s.query_realtime_start_s,
                 query_realtime_end_s=s.query_realtime_end_s)
        fatal = self.fatal_codes()
        r["fatal_errors"] = {k: v for k, v in r["errors"].items() if v.get("code") in fatal}
        return r

    def _power_fields(self, r: dict, s: Sample, caps: dict) -> None:
        """The four power fields (telemetry.py:119-193)."""
        r["memory_power_source"] = None
        missing = []
        for i, (key, field_name, _, scope_label) in enumerate(_POWER_SPECS):
            r[key] = None
            c = s.code[TF_POWER_INSTANT + i]
            if self.backend is not None and self.backend.table.field_missing[i]:
                err = self.error(self.backend.table.field_missing[i])
                r["errors"][key] = err
                caps[key] = {"available": False, "error": err}
                missing.append(i)
        if not s.flags & TS_FIELDS_QUERIED:
            r["memory_power_w"] = None
            return
        if s.code[TF_FIELD_QUERY]:
            err = self.error(s.code[TF_FIELD_QUERY])
            for i, (key, field_name, _, scope_label) in enumerate(_POWER_SPECS):
                if i in missing:
                    continue
                r["errors"][key] = err
                caps[key] = {"available": False, "field": field_name, "scope": scope_label, "error": err}
            r["memory_power_w"] = None
            return
        for i, (key, field_name, scope_name, scope_label) in enumerate(_POWER_SPECS):
            if i in missing:
                continue
            c = s.code[TF_POWER_INSTANT + i]
            if c:
                err = self.error(c, raw=s.field_value_type[i] if c == TE_VALUE_TYPE else self._field_raw(s, i))
                r["errors"][key] = err
                caps[key] = {"available": False, "field": field_name, "scope": scope_label, "error": err}
                continue
            scope_id = (self.backend.table.scope_id[i] if self.backend is not None else _NATIVE_SCOPES[scope_name])
            r["field_metadata"][key] = {
                "field": field_name, "scope": scope_label, "scope_id": scope_id,
                "timestamp_us": int(s.field_timestamp_us[i]), "timestamp_clock": "unix_epoch_microseconds",
                "latency_us": int(s.field_latency_us[i]),
                "semantics": "one_second_average" if "average" in key else "driver_instantaneous",
            }
            r[key] = s.field_mw[i] / 1000.0
            caps[key] = {"available": True, "field": field_name, "scope": scope_label}
        source = ("memory_power_instant_w" if r["memory_power_instant_w"] is not None
                  else "memory_power_average_w" if r["memory_power_average_w"] is not None else None)
        r["memory_power_w"] = r[source] if source else None
        r["memory_power_source"] = source
        caps["memory_power_w"] = {"available": source is not None, "source": source, "scope": "memory"}

    @staticmethod
    def _field_raw(s: Sample, i: int):
        v = s.field_mw[i]
        return int(v) if s.field_value_type[i] in (1, 2, 3, 4) and math.isfinite(v) and v == int(v) else v


# --------------------------------------------------------------------------- device
class NvmlDevice:
    """Select a physical NVML device by exact UUID (preferred) or NVML index.

    An NVML index is not a CUDA ordinal: CUDA_VISIBLE_DEVICES may reorder them.
    The caller must compare the benchmark's CUDA UUID to ``device.uuid``. MIG
    UUIDs are rejected because board power cannot be attributed to one slice.
    ``nvml_module`` replaces libnvidia-ml with a pynvml-like object.
    """

    def __init__(self, index: int = 0, uuid: str | None = None, nvml_module: Any = None):
        if uuid is not None and not uuid.startswith("GPU-"):
            raise TelemetryError("Use a complete physical GPU UUID beginning GPU-; MIG UUIDs are unsupported")
        lib = _lib()
        self.nvml = nvml_module
        self._backend = _ModuleBackend(nvml_module) if nvml_module is not None else None
        self.capabilities: dict[str, Any] = {}
        self._handle = _vp()
        table = None
        if self._backend is not None:
            self._backend.last_exception = None
            table = C.byref(self._backend.table)
        rc = lib.pm_nvml_open(table, int(index), uuid.encode() if uuid is not None else None, C.byref(self._handle))
        if rc:
            message = _last_error()
            exc = self._backend.last_exception if self._backend is not None else None
            if exc is not None and "failed with code" in message:
                raise exc
            raise TelemetryError(message)
        buf = C.create_string_buffer(96)
        lib.pm_nvml_uuid(self._handle, buf, len(buf))
        self.uuid = buf.value.decode()
        self.index = index if uuid is None else None
        self._closed = False
        self._convert = _Converter(self)

    @property
    def _active_samplers(self) -> int:
        return int(_lib().pm_nvml_active_samplers(self._handle))

    def read_sample(self) -> dict[str, Any]:
        sample = Sample()
        room = 3 * 4096
        procs = (Process * room)()
        rc = _lib().pm_nvml_read_sample(self._handle, C.byref(sample), procs, room)
        if rc:
            raise TelemetryError(_last_error())
        return self._convert.convert(sample, procs)

    sample = read_sample

    def metadata(self) -> dict[str, Any]:
        """Read metadata and probe monitoring capabilities without changing policy (telemetry.py:274-308)."""
        result: dict[str, Any] = {"uuid": self.uuid, "nvml_index": self.index, "errors": {}}
        if self._backend is not None:
            self._module_metadata(result)
        else:
            self._native_metadata(result)
        cc = result["compute_capability"]
        result["power_usage_semantics"] = (
            "instantaneous_device_and_associated_circuitry" if cc and (cc[0] < 8 or cc == [8, 0])
            else "one_second_average_device_and_associated_circuitry" if cc
            else "unknown_inspect_driver_and_architecture")
        result["energy_counter_units"] = "mJ_since_driver_reload"
        result["power_scope_note"] = ("Do not equate device/circuitry or GPU scope to an isolated core rail, or "
                                      "subtract a memory rail without validating scope inclusion on this SKU. No "
                                      "module-scope fallback is performed.")
        result["sample"] = self.read_sample()
        result["capabilities"] = dict(self.capabilities)
        result["capabilities"].update({
            "power_scope": "nvmlDeviceGetPowerUsage: device and associated circuitry (e.g. memory); driver/SKU "
                           "scope must be validated",
            "power_usage_semantics": result["power_usage_semantics"],
            "energy_counter_units": result["energy_counter_units"],
            "memory_power_source": result["sample"].get("memory_power_source"),
        })
        return result

    def _native_metadata(self, result: dict) -> None:
        m = Metadata()
        rc = _lib().pm_nvml_read_metadata(self._handle, C.byref(m))
        if rc:
            raise TelemetryError(_last_error())
        items = [
            ("name", "nvmlDeviceGetName", lambda: m.name.decode(errors="replace")),
            ("compute_capability", "nvmlDeviceGetCudaComputeCapability", lambda: [int(m.cc_major), int(m.cc_minor)]),
            ("memory", "nvmlDeviceGetMemoryInfo", lambda: {"total_bytes": int(m.memory_total),
                                                           "used_bytes": int(m.memory_used),
                                                           "free_bytes": int(m.memory_free)}),
            ("pci_bus_id", "nvmlDeviceGetPciInfo", lambda: m.pci_bus_id.decode(errors="replace")),
            ("mig_mode", "nvmlDeviceGetMigMode", lambda: {"current": int(m.mig_current), "pending": int(m.mig_pending)}),
            ("persistence_mode", "nvmlDeviceGetPersistenceMode", lambda: int(m.persistence_mode)),
            ("ecc_mode", "nvmlDeviceGetEccMode", lambda: {"current": int(m.ecc_current), "pending": int(m.ecc_pending)}),
            ("power_limit_constraints_w", "nvmlDeviceGetPowerManagementLimitConstraints",
             lambda: [m.power_limit_min_mw / 1000, m.power_limit_max_mw / 1000]),
            ("default_power_limit_w", "nvmlDeviceGetPowerManagementDefaultLimit",
             lambda: m.default_power_limit_mw / 1000),
        ]
        for slot, (key, api, value) in enumerate(items):
            if m.code[slot]:
                err = self._convert.error(m.code[slot])
                result[key] = None
                result["errors"][key] = err
                self.capabilities[key] = {"available": False, "api": api, "error": err}
            else:
                result[key] = value()
                self.capabilities[key] = {"available": True, "api": api}
        for slot, (key, text) in enumerate((("driver_version", m.driver_version), ("nvml_version", m.nvml_version)),
                                           start=9):
            if m.code[slot]:
                result[key] = None
                result["errors"][key] = self._convert.error(m.code[slot])
            else:
                result[key] = text.decode(errors="replace")

    def _module_metadata(self, result: dict) -> None:
        """Metadata through an injected module: the reference's reads, one call each."""
        nvml, handle = self.nvml, self._backend._handles[-1]

        def query(key, api, transform):
            try:
                result[key] = transform(getattr(nvml, api)(handle))
                self.capabilities[key] = {"available": True, "api": api}
            except Exception as exc:  # noqa: BLE001
                result[key] = None
                result["errors"][key] = _error(exc)
                self.capabilities[key] = {"available": False, "api": api, "error": _error(exc)}

        query("name", "nvmlDeviceGetName", _text)
        query("compute_capability", "nvmlDeviceGetCudaComputeCapability", lambda v: list(v))
        query("memory", "nvmlDeviceGetMemoryInfo",
              lambda v: {"total_bytes": int(v.total), "used_bytes": int(v.used), "free_bytes": int(v.free)})
        query("pci_bus_id", "nvmlDeviceGetPciInfo", lambda v: _text(v.busId))
        query("mig_mode", "nvmlDeviceGetMigMode", lambda v: {"current": int(v[0]), "pending": int(v[1])})
        query("persistence_mode", "nvmlDeviceGetPersistenceMode", int)
        query("ecc_mode", "nvmlDeviceGetEccMode", lambda v: {"current": int(v[0]), "pending": int(v[1])})
        query("power_limit_constraints_w", "nvmlDeviceGetPowerManagementLimitConstraints",
              lambda v: [v[0] / 1000, v[1] / 1000])
        query("default_power_limit_w", "nvmlDeviceGetPowerManagementDefaultLimit", lambda v: v / 1000)
        for key, api in (("driver_version", "nvmlSystemGetDriverVersion"), ("nvml_version", "nvmlSystemGetNVMLVersion")):
            try:
                result[key] = _text(getattr(nvml, api)())
            except Exception as exc:  # noqa: BLE001
                result[key] = None
                result["errors"][key] = _error(exc)

    def close(self) -> None:
        rc = _lib().pm_nvml_close(self._handle)
        if rc:
            raise TelemetryError(_last_error())
        self._closed = True

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()


# --------------------------------------------------------------------------- sampler
class Sampler:
    """Monotonic host sampling with explicit start/end bracket readings.

    The thread is native: one tick reads every sample field, the next deadline
    advances by ``interval_s`` and missed ticks are skipped; ``stop`` takes a
    final bracket sample on that thread.  A small polling interval does not
    increase the NVML sensor update rate.
    """

    def __init__(self, device: NvmlDevice, interval_s: float = 0.02):
        if not math.isfinite(interval_s) or interval_s < 0.001:
            raise ValueError("Telemetry interval must be finite and at least 0.001 seconds")
        self.device = device
        self.interval_s = float(interval_s)
        self._ptr = _vp()
        rc = _lib().pm_sampler_create(device._handle, self.interval_s, C.byref(self._ptr))
        if rc:
            raise TelemetryError(_last_error())
        self._cache: list[dict] = []
        self._procs = (Process * 0)()
        self._error: dict | None = None

    def _status(self):
        reason, where, running = C.c_int(), C.c_uint64(), C.c_int()
        _lib().pm_sampler_status(self._ptr, C.byref(reason), C.byref(where), C.byref(running))
        return reason.value, where.value, bool(running.value)

    @property
    def _attached(self) -> bool:
        return self._status()[2]

    @property
    def samples(self) -> list[dict]:
        lib = _lib()
        n, p = C.c_uint64(), C.c_uint64()
        lib.pm_sampler_count(self._ptr, C.byref(n), C.byref(p))
        have = len(self._cache)
        if n.value > have:
            fresh = (Sample * (n.value - have))()
            procs = (Process * max(1, p.value))()
            lib.pm_sampler_copy(self._ptr, have, n.value - have, fresh, procs, p.value)
            convert = self.device._convert
            self._cache.extend(convert.convert(s, procs) for s in fresh)
        return list(self._cache)

    @property
    def error(self) -> dict | None:
        if self._error is None:
            reason, where, _ = self._status()
            if reason == 1:
                samples = self.samples
                fatal = samples[where]["fatal_errors"] if where < len(samples) else {}
                self._error = {"type": "TelemetryError", "message": f"Fatal NVML device error: {fatal}"}
            elif reason == 3:
                self._error = {"type": "TelemetryError",
                               "message": "Another NVML query is still running; refusing concurrent driver access"}
        return self._error

    @error.setter
    def error(self, value: dict | None) -> None:
        self._error = value

    def start(self):
        rc = _lib().pm_sampler_start(self._ptr, 10.0)
        if rc == PM_E_NVML:
            raise TelemetryError(f"Initial NVML sample failed: {self.error}")
        if rc:
            raise TelemetryError(_last_error())
        return self

    def stop(self, timeout_s: float = 10) -> list[dict]:
        if not math.isfinite(timeout_s) or timeout_s <= 0:
            raise ValueError("Sampler shutdown timeout must be finite and positive")
        rc = _lib().pm_sampler_stop(self._ptr, float(timeout_s))
        if rc == PM_E_NVML:
            raise TelemetryError(f"NVML sampler failed: {self.error}")
        if rc:
            raise TelemetryError(_last_error())
        return self.samples

    def __enter__(self):
        return self.start()

    def __exit__(self, *_):
        self.stop()

    def __del__(self):
        ptr = getattr(self, "_ptr", None)
        if ptr:
            try:
                _lib().pm_sampler_destroy(ptr)
            except Exception:  # noqa: BLE001 - interpreter shutdown
                pass


class ClockWatch:
    """The SM clock and clock-event reasons read by a native thread every ``interval_s``
    (pm_clock_watch_*): many records even inside a timed region of milliseconds.

    ``stop()`` returns (t_s, sm_mhz, reason_bits) arrays of the successful reads."""

    def __init__(self, device: "NvmlDevice", interval_s: float = 1e-4):
        self.device, self.interval_s, self._ptr = device, interval_s, None

    def start(self) -> "ClockWatch":
        ptr = _vp()
        rc = _lib().pm_clock_watch_start(self.device._handle, self.interval_s, C.byref(ptr))
        if rc:
            raise TelemetryError(f"pm_clock_watch_start failed ({rc}): {_last_error()}")
        self._ptr = ptr
        return self

    def stop(self):
        import numpy as np
        if self._ptr is None:
            raise TelemetryError("clock watch not started")
        cap = 1 << 20
        mhz, bits = np.zeros(cap, np.uint32), np.zeros(cap, np.uint64)
        t, codes = np.zeros(cap, np.float64), np.zeros(cap, np.int32)
        count = C.c_uint64()
        rc = _lib().pm_clock_watch_stop(self._ptr, mhz.ctypes.data, bits.ctypes.data, t.ctypes.data, codes.ctypes.data,
                                        cap, C.byref(count))
        self._ptr = None
        if rc:
            raise TelemetryError(f"pm_clock_watch_stop failed ({rc}): {_last_error()}")
        n = count.value
        ok = codes[:n] == 0
        return t[:n][ok], mhz[:n][ok], bits[:n][ok]
