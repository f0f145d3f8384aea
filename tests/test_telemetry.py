"""Native NVML sampler against the reference's telemetry, on fake drivers (no GPU).

Golden samples and phase slices come from the reference's own NvmlDevice and
_phase_records run on the same scenarios (tests/golden/make_telemetry_golden.py).
"""
from __future__ import annotations

import gzip
import json
import math
import threading
import time
from pathlib import Path
from types import SimpleNamespace

import pytest

import nvml_fake
from nvml_fake import DriverError, FakeDriver
from powermodeling_b200.capture import phase_records
from powermodeling_b200.telemetry import NvmlDevice, Sampler, TelemetryError

GOLDEN = json.load(gzip.open(Path(__file__).parent / "golden" / "telemetry.json.gz", "rt"))


def clean(value):
    if isinstance(value, float) and math.isnan(value):
        return "nan"
    if isinstance(value, dict):
        return {k: clean(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [clean(v) for v in value]
    return value


@pytest.mark.parametrize("name", sorted(nvml_fake.SCENARIOS))
def test_read_sample_matches_reference(name):
    factory, reads = nvml_fake.SCENARIOS[name]
    golden = GOLDEN["samples"][name]
    fake = factory()
    with NvmlDevice(nvml_module=fake) as device:
        got = [nvml_fake.strip_timing(device.read_sample()) for _ in range(reads)]
        assert clean(got) == golden["reads"]
        assert clean(device.capabilities) == golden["capabilities"]
        meta = device.metadata()
        meta["sample"] = nvml_fake.strip_timing(meta["sample"])
        assert clean(meta) == golden["metadata"]


def test_sample_key_order_matches_reference():
    with NvmlDevice(nvml_module=FakeDriver(memory_rail=True)) as device:
        keys = list(device.read_sample())
    assert keys[:10] == ["uuid", "errors", "field_metadata", "power_w", "memory_power_source", "power_instant_w",
                         "power_average_w", "memory_power_instant_w", "memory_power_average_w", "memory_power_w"]
    assert keys[-7:] == ["t_s", "query_start_s", "query_end_s", "query_duration_s", "query_realtime_start_s",
                         "query_realtime_end_s", "fatal_errors"]


def test_timestamps_bracket_the_query():
    with NvmlDevice(nvml_module=FakeDriver()) as device:
        before = time.monotonic()
        s = device.read_sample()
        after = time.monotonic()
    assert before <= s["query_start_s"] <= s["t_s"] <= s["query_end_s"] <= after
    assert s["query_duration_s"] == pytest.approx(s["query_end_s"] - s["query_start_s"], abs=1e-12)
    assert s["query_realtime_start_s"] <= s["query_realtime_end_s"]
    assert abs(s["query_realtime_start_s"] - time.time()) < 5


@pytest.mark.parametrize("name", sorted(nvml_fake.phase_cases()))
def test_phase_records_match_reference(name):
    events, times = nvml_fake.phase_cases()[name]
    samples = [{"t_s": t, "i": i} for i, t in enumerate(times)]
    golden = GOLDEN["phases"][name]
    if "raises" in golden:
        with pytest.raises(ValueError) as info:
            phase_records(events, samples)
        assert [type(info.value).__name__, str(info.value)] == golden["raises"]
        return
    got = phase_records(events, samples)
    assert {k: {"start_s": v["start_s"], "end_s": v["end_s"], "samples": [s["i"] for s in v["samples"]]}
            for k, v in got.items()} == golden["phases"]


def test_phase_records_unordered_samples_follow_reference_slice():
    ns = 10 ** 9
    events = [{"type": "phase", "phase": "m", "event": "start", "host_monotonic_ns": 2 * ns},
              {"type": "phase", "phase": "m", "event": "end", "host_monotonic_ns": 3 * ns}]
    times = [1.0, 2.5, 5.0, 2.7, 0.5, 2.9, 4.0]
    samples = [{"t_s": t, "i": i} for i, t in enumerate(times)]
    got = [s["i"] for s in phase_records(events, samples)["m"]["samples"]]
    inside = [i for i, t in enumerate(times) if 2 <= t <= 3]
    assert got == list(range(max(0, inside[0] - 1), min(len(times), inside[-1] + 2)))


# ------------------------------------------------------------------ device selection and sessions
def test_uuid_selection_is_exact_and_mig_rejected():
    fake = FakeDriver()
    with NvmlDevice(uuid=fake.UUID, nvml_module=fake) as device:
        assert device.uuid == fake.UUID and device.index is None
        assert ("uuid_lookup", fake.UUID) in fake.events
        assert not any(isinstance(e, tuple) and e[0] == "index_lookup" for e in fake.events)
    with pytest.raises(TelemetryError, match="MIG UUIDs are unsupported"):
        NvmlDevice(uuid="MIG-abc", nvml_module=fake)
    with pytest.raises(TelemetryError, match="GPU UUID mismatch"):
        NvmlDevice(uuid="GPU-different", nvml_module=fake)


def test_mig_handle_rejected():
    fake = FakeDriver(uuid="MIG-1234")
    with pytest.raises(TelemetryError, match="Physical GPU handle required"):
        NvmlDevice(nvml_module=fake)
    assert fake.events.count("init") == fake.events.count("shutdown") == 1


def test_lookup_exception_propagates():
    fake = FakeDriver()

    def missing(index):
        raise DriverError(28, "GPU not found")
    fake.nvmlDeviceGetHandleByIndex = missing
    with pytest.raises(DriverError, match="GPU not found"):
        NvmlDevice(index=3, nvml_module=fake)


def test_shared_backend_not_shut_down_while_another_device_is_open():
    fake = FakeDriver()
    first = NvmlDevice(nvml_module=fake)
    second = NvmlDevice(nvml_module=fake)
    first.close()
    assert "shutdown" not in fake.events
    assert second.read_sample()["power_w"] == pytest.approx(612.345)
    second.close()
    assert fake.events.count("init") == 1 and fake.events.count("shutdown") == 1


def test_closed_device_refuses_reads():
    device = NvmlDevice(nvml_module=FakeDriver())
    device.close()
    device.close()
    with pytest.raises(TelemetryError, match="closed"):
        device.read_sample()


# ------------------------------------------------------------------ sampler
def test_sampler_brackets_order_and_close_protection():
    device = NvmlDevice(nvml_module=FakeDriver())
    sampler = Sampler(device, interval_s=0.002).start()
    with pytest.raises(TelemetryError, match="Stop all telemetry samplers"):
        device.close()
    time.sleep(0.02)
    samples = sampler.stop()
    assert len(samples) >= 3
    t = [s["t_s"] for s in samples]
    assert t == sorted(t)
    assert sampler.stop() == samples
    assert device._active_samplers == 0
    device.close()


def test_sampler_argument_checks():
    device = NvmlDevice(nvml_module=FakeDriver())
    for bad in (0.0005, math.nan, math.inf):
        with pytest.raises(ValueError, match="at least 0.001"):
            Sampler(device, interval_s=bad)
    sampler = Sampler(device, interval_s=0.01)
    with pytest.raises(TelemetryError, match="has not been started"):
        sampler.stop()
    sampler.start()
    with pytest.raises(TelemetryError, match="already been started"):
        sampler.start()
    with pytest.raises(ValueError, match="finite and positive"):
        sampler.stop(timeout_s=0)
    sampler.stop()
    device.close()


def test_fatal_first_sample_stops_sampler():
    fake = FakeDriver()

    def lost(handle):
        raise DriverError(15, "GPU lost")
    fake.nvmlDeviceGetPowerUsage = lost
    device = NvmlDevice(nvml_module=fake)
    sampler = Sampler(device, interval_s=0.001)
    with pytest.raises(TelemetryError, match="Initial NVML sample failed"):
        sampler.start()
    with pytest.raises(TelemetryError, match="NVML sampler failed"):
        sampler.stop()
    assert len(sampler.samples) == 1
    assert "power_w" in sampler.samples[0]["fatal_errors"]
    assert sampler.error["type"] == "TelemetryError" and "Fatal NVML device error" in sampler.error["message"]
    assert device._active_samplers == 0
    device.close()


def test_fatal_code_mid_run_ends_sampling_without_final_bracket():
    fake = FakeDriver()
    calls = {"n": 0}
    original = fake.nvmlDeviceGetPowerUsage

    def failing(handle):
        calls["n"] += 1
        if calls["n"] >= 5:
            raise DriverError(16, "Reset required")
        return original(handle)
    fake.nvmlDeviceGetPowerUsage = failing
    device = NvmlDevice(nvml_module=fake)
    sampler = Sampler(device, interval_s=0.001).start()
    deadline = time.monotonic() + 5
    while sampler._attached and time.monotonic() < deadline:
        time.sleep(0.005)
    assert not sampler._attached
    with pytest.raises(TelemetryError, match="NVML sampler failed"):
        sampler.stop()
    samples = sampler.samples
    assert len(samples) == 5 and samples[-1]["fatal_errors"]["power_w"]["code"] == 16
    assert not any(s["fatal_errors"] for s in samples[:-1])
    device.close()


def test_non_fatal_errors_keep_sampling():
    fake = FakeDriver()

    def flaky(handle):
        raise DriverError(3, "Not Supported")
    fake.nvmlDeviceGetPowerUsage = flaky
    device = NvmlDevice(nvml_module=fake)
    sampler = Sampler(device, interval_s=0.002).start()
    time.sleep(0.03)
    samples = sampler.stop()
    assert len(samples) >= 3 and all(s["power_w"] is None and not s["fatal_errors"] for s in samples)
    device.close()


def test_stuck_query_cannot_block_stop_or_unsafe_close():
    fake = FakeDriver()
    entered, release = threading.Event(), threading.Event()
    original = fake.nvmlDeviceGetPowerUsage
    queries = {"n": 0}

    def block_second(handle):
        queries["n"] += 1
        if queries["n"] == 2:
            entered.set()
            release.wait(timeout=2)
        return original(handle)
    fake.nvmlDeviceGetPowerUsage = block_second
    device = NvmlDevice(nvml_module=fake)
    sampler = Sampler(device, interval_s=0.001).start()
    try:
        assert entered.wait(timeout=1)
        started = time.monotonic()
        with pytest.raises(TelemetryError, match="did not stop"):
            sampler.stop(timeout_s=0.002)
        with pytest.raises(TelemetryError, match="Stop all telemetry samplers"):
            device.close()
        assert time.monotonic() - started < 0.1
        assert "shutdown" not in fake.events
    finally:
        release.set()
        samples = sampler.stop(timeout_s=2)
        device.close()
    assert len(samples) == 3  # first, the stuck tick, and the final bracket


def test_missed_ticks_are_skipped_not_caught_up():
    fake = FakeDriver()
    original = fake.nvmlDeviceGetPowerUsage

    def slow(handle):
        time.sleep(0.012)
        return original(handle)
    fake.nvmlDeviceGetPowerUsage = slow
    device = NvmlDevice(nvml_module=fake)
    sampler = Sampler(device, interval_s=0.002).start()
    time.sleep(0.15)
    samples = sampler.stop()
    device.close()
    starts = [s["query_start_s"] for s in samples]
    gaps = [b - a for a, b in zip(starts, starts[1:])]
    # every query takes >= 12 ms; a catch-up loop would start the next one at once,
    # the skip rule waits for a fresh interval after the slow query ends
    assert len(samples) <= 0.15 / 0.012 + 3
    assert min(gaps[:-1]) >= 0.012 + 0.001


def test_tick_rate_at_5_ms():
    device = NvmlDevice(nvml_module=FakeDriver())
    sampler = Sampler(device, interval_s=0.005).start()
    time.sleep(0.3)
    samples = sampler.stop()
    device.close()
    assert 30 <= len(samples) <= 70
    starts = [s["query_start_s"] for s in samples]
    assert all(b > a for a, b in zip(starts, starts[1:]))


def test_energy_counter_decrease_flagged_in_sampler_stream():
    fake = FakeDriver()
    fake.energy = [100, 200, 50, 60]
    device = NvmlDevice(nvml_module=fake)
    samples = [device.read_sample() for _ in range(4)]
    device.close()
    assert [s["energy_counter_decreased"] for s in samples] == [False, False, True, False]
    assert samples[2]["errors"]["energy_counter"]["type"] == "CounterDecrease"


def test_process_list_grows_beyond_the_first_buffer():
    fake = FakeDriver()
    fake.processes = [SimpleNamespace(pid=10 + i, usedGpuMemory=i) for i in range(300)]
    device = NvmlDevice(nvml_module=fake)
    sampler = Sampler(device, interval_s=0.005).start()
    time.sleep(0.02)
    samples = sampler.stop()
    device.close()
    assert all(len(s["compute_processes"]) == 300 for s in samples)
    assert samples[-1]["compute_processes"][299] == {"pid": 309, "used_gpu_memory_bytes": 299}


def test_native_backend_without_a_driver_fails_cleanly():
    try:
        device = NvmlDevice()
    except TelemetryError as exc:
        assert "NVML" in str(exc)
        return
    device.close()
    pytest.skip("a driver is present: the native backend opened a real device")


def test_capture_without_a_gpu_keeps_samples_and_reports_failure():
    from powermodeling_b200.capture import capture_trial
    device = NvmlDevice(nvml_module=FakeDriver())
    record = capture_trial(["--workload", "hbm", "--seconds", "1"], device, sample_interval_s=0.005)
    device.close()
    q = record["quality"]
    assert q["benchmark_exit_code"] == 1 and any("powerbench failed" in e for e in q["runner_errors"])
    assert record["status"] == "failed" and len(record["samples"]) >= 2
    assert record["device"]["name"] == "NVIDIA B200" and record["telemetry"]["power_w"]["available"]


def test_clock_watch_reads_the_sm_clock_and_reasons_on_its_own_thread():
    import time
    from powermodeling_b200.telemetry import ClockWatch
    from nvml_fake import FakeDriver
    with NvmlDevice(nvml_module=FakeDriver()) as device:
        watch = ClockWatch(device, interval_s=0.001).start()
        try:
            attached = device._active_samplers
            time.sleep(0.05)
        finally:
            t, mhz, bits = watch.stop()
        assert attached == 1 and device._active_samplers == 0
        ref = device.read_sample()
    assert 10 <= len(t) <= 80
    assert (t[1:] > t[:-1]).all()
    assert set(mhz.tolist()) == {ref["sm_clock_mhz"]}
    assert set(bits.tolist()) == {ref["throttle_reasons"]}
