"""The native NVML sampler on a real B200, and one captured trial through the GPU analysis."""
from __future__ import annotations

import time

import pytest

from conftest import close, diff
from oracle import analysis_oracle as O
from tests.golden.make_golden import TRIAL_KEYS

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def device(gpu_ready):
    from powermodeling_b200 import powerbench
    from powermodeling_b200.telemetry import NvmlDevice
    cuda = next(r for r in powerbench.run(["--describe"]) if r["type"] == "device")
    dev = NvmlDevice(uuid=cuda["uuid"])
    yield dev
    dev.close()


def test_live_sample_schema_and_values(device):
    s = device.read_sample()
    assert s["uuid"] == device.uuid and s["uuid"].startswith("GPU-")
    assert not s["fatal_errors"]
    assert 20 < s["power_w"] < 1500
    assert s["energy_mj"] > 0 and s["energy_counter_decreased"] is False
    assert s["sm_clock_mhz"] > 0 and s["memory_clock_mhz"] > 0 and s["graphics_clock_mhz"] > 0
    assert 0 < s["power_limit_w"] <= 1500 and 0 < s["enforced_power_limit_w"] <= 1500
    assert isinstance(s["throttle_reason_names"], list)
    assert s["power_instant_w"] is None or 20 < s["power_instant_w"] < 1500
    assert isinstance(s["compute_processes"], list)
    assert s["query_start_s"] <= s["t_s"] <= s["query_end_s"]
    meta = device.metadata()
    assert meta["compute_capability"] == [10, 0]
    assert meta["power_usage_semantics"] == "one_second_average_device_and_associated_circuitry"
    assert "B200" in meta["name"] and meta["memory"]["total_bytes"] > 100e9


def test_native_reads_agree_with_pynvml(device):
    pynvml = pytest.importorskip("pynvml")
    pynvml.nvmlInit()
    try:
        h = pynvml.nvmlDeviceGetHandleByUUID(device.uuid)
        s = device.read_sample()
        assert s["power_limit_w"] == pynvml.nvmlDeviceGetPowerManagementLimit(h) / 1000
        assert s["enforced_power_limit_w"] == pynvml.nvmlDeviceGetEnforcedPowerLimit(h) / 1000
        assert s["memory_clock_mhz"] == pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_MEM)
        e0 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h)
        s2 = device.read_sample()
        e1 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h)
        assert e0 <= s2["energy_mj"] <= e1
        bus = pynvml.nvmlDeviceGetPciInfo(h).busId
        assert device.metadata()["pci_bus_id"] == (bus.decode() if isinstance(bus, bytes) else bus)
    finally:
        pynvml.nvmlShutdown()


def test_sampler_10ms_ticks(device):
    from powermodeling_b200.telemetry import Sampler
    sampler = Sampler(device, interval_s=0.01).start()
    time.sleep(1.0)
    samples = sampler.stop()
    # A full sample makes every reference read; the driver sets its cost (the
    # energy-counter read alone took 4 ms p50 to 24 ms max on B200 boxes), and
    # missed 10 ms ticks are skipped.  So the cadence is checked against the
    # samples' own query times: the next query starts by the first tick after
    # the previous one ended (plus scheduling slack), and no tick is doubled.
    assert 5 <= len(samples) <= 110
    starts = [s["query_start_s"] for s in samples]
    for prev, cur, d in zip(starts, starts[1:], (s["query_duration_s"] for s in samples)):
        assert cur - prev <= d + 0.010 + 0.005, (prev, cur, d)
    busy = sum(s["query_duration_s"] for s in samples)
    assert len(samples) >= 0.5 * (starts[-1] - starts[0]) / (0.010 + busy / len(samples))
    t = [s["t_s"] for s in samples]
    assert all(b > a for a, b in zip(t, t[1:]))
    energy = [s["energy_mj"] for s in samples]
    assert all(b >= a for a, b in zip(energy, energy[1:]))
    assert not any(s["fatal_errors"] for s in samples)


def test_captured_hbm_trial_analysis_matches_oracle(device):
    """A real 2 s HBM read under the 10 ms sampler: phases, then the GPU analysis against the oracle."""
    from powermodeling_b200.analysis import analyze_trial
    from powermodeling_b200.capture import capture_trial
    from powermodeling_b200.synthetic import ANALYSIS_POLICY
    args = ["--workload", "hbm", "--memory-vector-bytes", "16", "--read-cache-policy", "cs",
            "--working-set-bytes", 1 << 30, "--blocks", 148 * 4, "--threads", 256, "--iterations", 256,
            "--seconds", 2, "--warmup-seconds", 0.5, "--idle-seconds", 1]
    record = capture_trial(args, device, sample_interval_s=0.01)
    assert record["quality"]["benchmark_exit_code"] == 0, record["quality"]["runner_errors"]
    assert not record["quality"]["runner_errors"], record["quality"]["runner_errors"]
    phases = record["phases"]
    assert {"idle_pre", "measure", "idle_post"} <= set(phases)
    measure = phases["measure"]
    assert len(measure["samples"]) >= 40   # ~20 samples/s at least: the energy-counter read slows under load
    assert measure["samples"][0]["t_s"] <= measure["start_s"] and measure["samples"][-1]["t_s"] >= measure["end_s"]
    assert record["benchmark"]["measure_epochs"]
    got = analyze_trial(record, ANALYSIS_POLICY)
    expected = O.analyze(record, ANALYSIS_POLICY)
    problems = diff(expected, got, TRIAL_KEYS, rel=1e-6)
    assert not problems, problems
    for key in ("total_energy_j", "board_power_w", "idle_power_w", "incremental_energy_j", "pj_per_logical_byte"):
        assert close(expected.get(key), got.get(key), rel=0.0), (key, expected.get(key), got.get(key))
    assert got["board_power_w"] > got["idle_power_w"] > 0
    assert got["total_energy_j"] > 0


def test_captured_nonlinear_trial_analysis_matches_oracle(device):
    """A captured RMSNorm trial (complete nonlinear function, Q-grid record) through the same path:
    the record passes the count contract and its per-element and per-row energies match the oracle."""
    from powermodeling_b200.analysis import analyze_trial
    from powermodeling_b200.capture import capture_trial
    from powermodeling_b200.contracts import nonlinear_count_issues
    from powermodeling_b200.synthetic import ANALYSIS_POLICY
    args = ["--workload", "rmsnorm", "--nonlinear-mode", "streaming", "--row-width", 1024, "--grid-mode", "fixed",
            "--blocks", 148 * 8, "--threads", 256, "--working-set-bytes", 1 << 30,
            "--seconds", 2, "--warmup-seconds", 0.5, "--idle-seconds", 1]
    record = capture_trial(args, device, sample_interval_s=0.01)
    assert record["quality"]["benchmark_exit_code"] == 0, record["quality"]["runner_errors"]
    assert not record["quality"]["runner_errors"], record["quality"]["runner_errors"]
    assert nonlinear_count_issues(record["benchmark"], "rmsnorm") == []
    got = analyze_trial(record, ANALYSIS_POLICY)
    expected = O.analyze(record, ANALYSIS_POLICY)
    problems = diff(expected, got, TRIAL_KEYS, rel=1e-6)
    assert not problems, problems
    for key in ("total_energy_j", "board_power_w", "idle_power_w", "throughput_elements_s", "total_pj_per_element",
                "total_pj_per_row"):
        assert close(expected.get(key), got.get(key), rel=0.0), (key, expected.get(key), got.get(key))
    assert not [i for i in got["issues"] if "nonlinear" in i], got["issues"]
    assert got["throughput_elements_s"] > 1e11 and got["total_pj_per_element"] > 0


def test_captured_paired_softmax_trial(device):
    """A captured softmax trial with the paired active reference (the reference's minimum arms: 10 s,
    1 s warm-up, 6 s idles): the engine's no-admission issue-loop record matches the treatment's
    geometry, the paired checks raise nothing, and the paired per-element energy equals the oracle's."""
    from powermodeling_b200.analysis import analyze_trial
    from powermodeling_b200.capture import capture_trial
    args = ["--workload", "softmax", "--nonlinear-mode", "streaming", "--row-width", 1024, "--grid-mode", "fixed",
            "--blocks", 148 * 8, "--threads", 256, "--working-set-bytes", 1 << 28, "--paired-reference",
            "--reference-order", "BA", "--seconds", 10, "--warmup-seconds", 1, "--idle-seconds", 6]
    record = capture_trial(args, device, sample_interval_s=0.01)
    assert record["quality"]["benchmark_exit_code"] == 0, record["quality"]["runner_errors"]
    ref = record["active_reference"]
    assert ref["kernel_implementation_version"] == "integer_issue_loop_no_admission_v2"
    for key in ("blocks", "threads", "batch_launches", "iterations_per_launch"):
        assert ref[key] == record["benchmark"][key], key
    assert ref["admitted_blocks"] == ref["batches"] * ref["batch_launches"] * ref["blocks"]
    got = analyze_trial(record)
    expected = O.analyze(record)
    problems = diff(expected, got, TRIAL_KEYS, rel=1e-6)
    assert not problems, problems
    assert not [i for i in got["paired_active_reference_issues"] if i.startswith("paired_protocol")
                or i.startswith("paired_geometry") or "definition" in i], got["paired_active_reference_issues"]
    assert got["throughput_elements_s"] > 1e11
    for key in ("paired_active_reference_power_w", "paired_active_reference_pj_per_element"):
        assert close(expected.get(key), got.get(key), rel=0.0), (key, expected.get(key), got.get(key))
