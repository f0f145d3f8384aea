"""A pynvml-like fake driver for hardware-free telemetry tests, and the scenarios built on it.

The same scenario objects drive the reference's NvmlDevice (to write the
golden samples, tests/golden/make_telemetry_golden.py) and this package's
native sampler (tests/test_telemetry.py).
"""
from __future__ import annotations

import math
import threading
from types import SimpleNamespace


class FakeDriver:
    """Driver surface: UUID/index lookup, power fields, energy, clocks, limits, processes."""

    NVML_CLOCK_GRAPHICS = 0
    NVML_CLOCK_SM = 1
    NVML_CLOCK_MEM = 2
    NVML_TEMPERATURE_GPU = 0
    NVML_POWER_SCOPE_GPU = 0
    NVML_POWER_SCOPE_MEMORY = 2
    NVML_FI_DEV_POWER_INSTANT = 186
    NVML_FI_DEV_POWER_AVERAGE = 185
    NVML_VALUE_TYPE_DOUBLE = 0
    NVML_VALUE_TYPE_UNSIGNED_INT = 1
    NVML_SUCCESS = 0
    nvmlClocksThrottleReasonSwPowerCap = 4
    nvmlClocksThrottleReasonHwSlowdown = 8
    nvmlClocksThrottleReasonGpuIdle = 1

    UUID = "GPU-0b200000-1111-2222-3333-444455556666"

    def __init__(self, cc=(10, 0), memory_rail=False, uuid=None):
        self.cc = cc
        self.memory_rail = memory_rail
        self.uuid = uuid or self.UUID
        self.energy = [5_000_000]
        self.power_mw = 612_345
        self.field_mw = {(186, 0): 598_000, (185, 0): 601_250, (186, 2): 91_500, (185, 2): 90_125}
        self.field_type = 1
        self.field_timestamp = 1_764_000_000_123_456
        self.field_latency = 25
        self.throttle = 4
        self.processes = [SimpleNamespace(pid=4242, usedGpuMemory=None)]
        self.events = []
        self.field_hook = None
        self.calls = 0
        self.lock = threading.Lock()

    # lifecycle
    def nvmlInit(self):
        self.events.append("init")

    def nvmlShutdown(self):
        self.events.append("shutdown")

    def nvmlDeviceGetHandleByUUID(self, uuid):
        self.events.append(("uuid_lookup", uuid))
        return ("handle", uuid)

    def nvmlDeviceGetHandleByIndex(self, index):
        self.events.append(("index_lookup", index))
        return ("handle", index)

    def nvmlDeviceGetUUID(self, handle):
        return self.uuid.encode()

    # metadata
    def nvmlDeviceGetName(self, handle):
        return b"NVIDIA B200"

    def nvmlDeviceGetCudaComputeCapability(self, handle):
        return self.cc

    def nvmlDeviceGetMemoryInfo(self, handle):
        return SimpleNamespace(total=192_000_000_000, used=1_000_000, free=191_999_000_000)

    def nvmlDeviceGetPciInfo(self, handle):
        return SimpleNamespace(busId=b"00000000:1B:00.0")

    def nvmlDeviceGetPowerManagementLimitConstraints(self, handle):
        return (200_000, 1_000_000)

    def nvmlDeviceGetPowerManagementDefaultLimit(self, handle):
        return 1_000_000

    def nvmlSystemGetDriverVersion(self):
        return "580.159"

    # sample reads
    def nvmlDeviceGetPowerUsage(self, handle):
        with self.lock:
            self.calls += 1
        return self.power_mw

    def nvmlDeviceGetFieldValues(self, handle, fields):
        out = []
        for field_id, scope in fields:
            unsupported = scope == self.NVML_POWER_SCOPE_MEMORY and not self.memory_rail
            out.append(SimpleNamespace(
                nvmlReturn=3 if unsupported else 0, valueType=self.field_type,
                value=SimpleNamespace(uiVal=self.field_mw[(field_id, scope)],
                                      dVal=float(self.field_mw[(field_id, scope)])),
                timestamp=self.field_timestamp, latencyUsec=self.field_latency))
        if self.field_hook is not None:
            out = self.field_hook(fields, out)
        return out

    def nvmlDeviceGetTotalEnergyConsumption(self, handle):
        value = self.energy[0]
        if len(self.energy) > 1:
            self.energy.pop(0)
        return value

    def nvmlDeviceGetClockInfo(self, handle, clock):
        return {0: 1965, 1: 1965, 2: 3996}[clock]

    def nvmlDeviceGetTemperature(self, handle, sensor):
        return 54

    def nvmlDeviceGetPerformanceState(self, handle):
        return 0

    def nvmlDeviceGetCurrentClocksThrottleReasons(self, handle):
        return self.throttle

    def nvmlDeviceGetUtilizationRates(self, handle):
        return SimpleNamespace(gpu=100, memory=87)

    def nvmlDeviceGetPowerManagementLimit(self, handle):
        return 1_000_000

    nvmlDeviceGetEnforcedPowerLimit = nvmlDeviceGetPowerManagementLimit

    def nvmlDeviceGetComputeRunningProcesses(self, handle):
        return list(self.processes)

    def nvmlDeviceGetGraphicsRunningProcesses(self, handle):
        return []


class DriverError(RuntimeError):
    """An error carrying an NVML-style ``value`` code, like pynvml's NVMLError."""

    def __init__(self, value, text="driver error"):
        super().__init__(text)
        self.value = value


class WithErrorClass(FakeDriver):
    """A driver that also exports an NVMLError class and MPS process reads."""

    class NVMLError(Exception):
        def __init__(self, value):
            super().__init__(f"NVML error {value}")
            self.value = value

    NVML_ERROR_GPU_IS_LOST = 15
    nvmlClocksEventReasonSwPowerCap = 4
    nvmlClocksEventReasonSyncBoost = 16

    def nvmlDeviceGetMPSComputeRunningProcesses(self, handle):
        return [SimpleNamespace(pid=77, usedGpuMemory=(1 << 64) - 1)]

    def nvmlDeviceGetCurrentClocksEventReasons(self, handle):
        return 4 | 16 | 1


class NoMemoryScope(FakeDriver):
    """A driver without the memory power-scope constant."""

    def __getattribute__(self, name):
        if name == "NVML_POWER_SCOPE_MEMORY":
            raise AttributeError(f"'NoMemoryScope' object has no attribute '{name}'")
        return super().__getattribute__(name)


def _memory_average_only(fake):
    def hook(fields, out):
        for value, (field_id, scope) in zip(out, fields):
            value.fieldId, value.scopeId = field_id, scope
            if scope == 2:
                if field_id == 186:
                    value.nvmlReturn = 3
                else:
                    value.value.uiVal = 43_125
                    value.timestamp, value.latencyUsec = 1_730_000_000_123_456, 35
        return out
    fake.field_hook = hook
    return fake


def _bad_metadata(field_id, attribute):
    def make():
        fake = FakeDriver(memory_rail=True)

        def hook(fields, out):
            for value, (requested, scope) in zip(out, fields):
                if scope == 2:
                    if requested == field_id:
                        setattr(value, attribute, "invalid sensor metadata")
                    else:
                        value.nvmlReturn = 3
            return out
        fake.field_hook = hook
        return fake
    return make


def _field_hook(fn, **kw):
    def make():
        fake = FakeDriver(**kw)
        fake.field_hook = fn
        return fake
    return make


def _set(**attrs):
    def make():
        fake = FakeDriver(memory_rail=attrs.pop("memory_rail", False))
        for k, v in attrs.items():
            setattr(fake, k, v)
        return fake
    return make


def _raising(method, exc_factory, base=FakeDriver):
    def make():
        fake = base()

        def fail(*args):
            raise exc_factory()
        setattr(fake, method, fail)
        return fake
    return make


def _wrong(attr, value):
    def hook(fields, out):
        for v, (field_id, scope) in zip(out, fields):
            v.fieldId, v.scopeId = field_id, scope
            setattr(v, attr, value)
        return out
    return hook


def _typed(value_type, ui=None, d=None):
    def hook(fields, out):
        for v in out:
            v.valueType = value_type
            if ui is not None:
                v.value.uiVal = ui
            if d is not None:
                v.value.dVal = d
        return out
    return hook


def _short(fields, out):
    return out[:-1]


# name -> (factory, reads): each scenario is read ``reads`` times in a row.
SCENARIOS = {
    "base": (FakeDriver, 1),
    "hopper_cc": (lambda: FakeDriver(cc=(9, 0)), 1),
    "memory_rail": (lambda: FakeDriver(memory_rail=True), 1),
    "memory_average_only": (lambda: _memory_average_only(FakeDriver(memory_rail=True)), 1),
    "bad_meta_instant_timestamp": (_bad_metadata(186, "timestamp"), 1),
    "bad_meta_instant_latency": (_bad_metadata(186, "latencyUsec"), 1),
    "bad_meta_average_timestamp": (_bad_metadata(185, "timestamp"), 1),
    "bad_meta_average_latency": (_bad_metadata(185, "latencyUsec"), 1),
    "power_usage_raises": (_raising("nvmlDeviceGetPowerUsage", lambda: RuntimeError("sensor not supported")), 1),
    "energy_decrease": (_set(energy=[(1 << 54) + 1, 10, 12]), 3),
    "energy_negative": (_set(energy=[-1]), 1),
    "energy_fraction": (_set(energy=[1.5]), 1),
    "energy_bool": (_set(energy=[True]), 1),
    "wrong_scope": (_field_hook(_wrong("scopeId", 0), memory_rail=True), 1),
    "wrong_field_id": (_field_hook(_wrong("fieldId", 999), memory_rail=True), 1),
    "short_field_list": (_field_hook(_short, memory_rail=True), 1),
    "field_query_raises": (_raising("nvmlDeviceGetFieldValues", lambda: DriverError(2, "Invalid Argument")), 1),
    "gpu_lost": (_raising("nvmlDeviceGetPowerUsage", lambda: DriverError(15, "GPU lost")), 1),
    "no_memory_scope": (NoMemoryScope, 1),
    "process_pid_zero": (_set(processes=[SimpleNamespace(pid=0, usedGpuMemory=5)]), 1),
    "process_used_bytes": (_set(processes=[SimpleNamespace(pid=9, usedGpuMemory=123_456),
                                           SimpleNamespace(pid=10, usedGpuMemory=(1 << 64) - 1)]), 1),
    "many_processes": (_set(processes=[SimpleNamespace(pid=1000 + i, usedGpuMemory=i) for i in range(150)]), 1),
    "throttle_bits": (_set(throttle=4 | 8 | 1 | 2), 1),
    "double_fields": (_field_hook(_typed(0, d=512_250.5), memory_rail=True), 1),
    "negative_double_field": (_field_hook(_typed(0, d=-3.0), memory_rail=True), 1),
    "nan_double_field": (_field_hook(_typed(0, d=math.nan)), 1),
    "unsupported_value_type": (_field_hook(_typed(9)), 1),
    "negative_power_limit": (_set(nvmlDeviceGetPowerManagementLimit=lambda h: -5), 1),
    "float_power": (_set(power_mw=612_345.75), 1),
    "error_class_driver": (WithErrorClass, 1),
    "error_class_gpu_lost_field": (lambda: _error_class_field(15), 1),
    "error_class_not_supported_field": (lambda: _error_class_field(3), 1),
}


def _error_class_field(code):
    fake = WithErrorClass(memory_rail=True)

    def hook(fields, out):
        out[0].nvmlReturn = code
        return out
    fake.field_hook = hook
    return fake


# Keys whose values are host timestamps (they differ between any two reads).
TIMING_KEYS = ("t_s", "query_start_s", "query_end_s", "query_duration_s", "query_realtime_start_s",
               "query_realtime_end_s")


def strip_timing(sample: dict) -> dict:
    return {k: v for k, v in sample.items() if k not in TIMING_KEYS}


# Phase slicing cases: (events, sample times).
def phase_cases():
    ns = 1_000_000_000
    t = [0.5 + 0.01 * i for i in range(400)]

    def ev(phase, kind, s):
        return {"type": "phase", "phase": phase, "event": kind, "host_monotonic_ns": int(round(s * ns))}

    return {
        "three_phases": ([ev("idle_pre", "start", 0.6), ev("idle_pre", "end", 1.1), ev("measure", "start", 1.2),
                          ev("measure", "end", 3.2), ev("idle_post", "start", 3.3), ev("idle_post", "end", 4.3),
                          {"type": "result"}], t),
        "phase_before_samples": ([ev("early", "start", 0.1), ev("early", "end", 0.2)], t),
        "edges_on_samples": ([ev("measure", "start", 1.0), ev("measure", "end", 2.0)], t),
        "first_sample_inside": ([ev("measure", "start", 0.4), ev("measure", "end", 0.8)], t),
        "last_sample_inside": ([ev("measure", "start", 4.0), ev("measure", "end", 9.0)], t),
        "no_samples": ([ev("measure", "start", 1.0), ev("measure", "end", 2.0)], []),
        "duplicate_start": ([ev("measure", "start", 1.0), ev("measure", "start", 1.5), ev("measure", "end", 2.0)], t),
        "end_before_start": ([ev("measure", "start", 2.0), ev("measure", "end", 1.0)], t),
        "missing_end": ([ev("measure", "start", 1.0)], t),
        "bad_kind": ([{"type": "phase", "phase": "measure", "event": "middle", "host_monotonic_ns": 5}], t),
        "negative_stamp": ([{"type": "phase", "phase": "measure", "event": "start", "host_monotonic_ns": -1}], t),
        "bool_stamp": ([{"type": "phase", "phase": "measure", "event": "start", "host_monotonic_ns": True}], t),
        "float_stamp": ([{"type": "phase", "phase": "measure", "event": "start", "host_monotonic_ns": 1.5}], t),
        "empty_name": ([{"type": "phase", "phase": "", "event": "start", "host_monotonic_ns": 5}], t),
        "non_dict_event": ([["phase"]], t),
        "bad_sample_time": ([ev("measure", "start", 1.0), ev("measure", "end", 2.0)], t[:3] + [math.nan]),
    }
