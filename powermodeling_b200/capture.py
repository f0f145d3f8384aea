"""Phase slicing of telemetry samples, and an in-process trial capture.

``phase_records`` restates powermodeling/runner.py ``_phase_records``
(177-205): phase events from powerbench (``host_monotonic_ns``, the same
CLOCK_MONOTONIC the sampler stamps ``t_s`` with) become
``{name: {start_s, end_s, samples}}`` where ``samples`` holds every sample
inside ``[start_s, end_s]`` plus one neighbour on each side, so the energy
integral can interpolate at the window edges without extrapolating.

``capture_trial`` is the measurement loop around one powerbench run: device
metadata, the native sampler started before and stopped after the run,
powerbench executed in this process (libpmb200's engine), and the record
fields the analysis reads (``benchmark``, ``active_reference``,
``treatment_protocol``, ``phases``, ``samples``, ``device``,
``cuda_device``, ``quality.measurement_pid``).  The reference's planner,
clock policy and exclusivity bookkeeping around it (runner.py:331-470) are
not part of this path.
"""
from __future__ import annotations

import bisect
import math
import os
from typing import Any

from . import powerbench
from .telemetry import NvmlDevice, Sampler


def phase_records(events: list, samples: list) -> dict[str, dict[str, Any]]:
    """Phases with their samples and one neighbour on each side (runner.py:177-205)."""
    phases: dict[str, dict[str, Any]] = {}
    for event in events:
        if not isinstance(event, dict):
            raise ValueError("Benchmark events must be JSON objects")
        if event.get("type") != "phase":
            continue
        name, kind = event.get("phase"), event.get("event")
        stamp = event.get("host_monotonic_ns")
        if (not isinstance(name, str) or not name or kind not in ("start", "end")
                or not isinstance(stamp, int) or isinstance(stamp, bool) or stamp < 0):
            raise ValueError("Malformed benchmark phase event")
        phase = phases.setdefault(name, {})
        key = "start_s" if kind == "start" else "end_s"
        if key in phase:
            raise ValueError(f"Duplicate {name} {kind} event")
        phase[key] = stamp / 1e9
    times = None
    for phase in phases.values():
        start, end = phase.get("start_s"), phase.get("end_s")
        if start is None or end is None or end <= start:
            raise ValueError("Benchmark phase must have increasing start/end timestamps")
        if times is None:
            if any(not isinstance(s, dict) or not isinstance(s.get("t_s"), (int, float))
                   or not math.isfinite(s["t_s"]) for s in samples):
                raise ValueError("Telemetry sample must have a finite monotonic timestamp")
            times = [s["t_s"] for s in samples]
            ordered = all(a <= b for a, b in zip(times, times[1:]))
        if ordered:
            first = bisect.bisect_left(times, start)
            last = bisect.bisect_right(times, end) - 1
            inside = (first, last) if first <= last else None
        else:
            hits = [i for i, t in enumerate(times) if start <= t <= end]
            inside = (hits[0], hits[-1]) if hits else None
        if inside:
            lo, hi = max(0, inside[0] - 1), min(len(samples), inside[1] + 2)
            phase["samples"] = samples[lo:hi]
        else:
            phase["samples"] = []
    return phases


def capture_trial(args: list, device: NvmlDevice, sample_interval_s: float = 0.01,
                  config: dict | None = None, trial_id: str | None = None) -> dict[str, Any]:
    """Runs powerbench ``args`` in this process under the native sampler; returns the trial record.

    ``status`` is "complete" when the capture raised no runner error, as the
    reference's runner marks a trial (runner.py:476); ``trial_id`` is the
    plan's id for the trial (analysis reports a trial without one)."""
    record: dict[str, Any] = {
        "schema_version": 1, "trial_id": trial_id, "status": "failed", "config": dict(config or {}),
        "benchmark": {}, "active_reference": {}, "treatment_protocol": {}, "phases": {}, "samples": [],
        "events": [], "device": {}, "cuda_device": {}, "telemetry": {},
        "quality": {"valid": False, "benchmark_exit_code": None, "runner_errors": [],
                    "measurement_pid": os.getpid()},
    }
    record["config"]["sample_interval_s"] = sample_interval_s
    quality = record["quality"]
    record["device"] = device.metadata()
    record["telemetry"] = record["device"].get("capabilities", {})
    sampler = Sampler(device, interval_s=sample_interval_s).start()
    try:
        events = powerbench.run([str(a) for a in args])
        quality["benchmark_exit_code"] = 0
    except powerbench.PowerbenchError as exc:
        events = exc.records
        quality["benchmark_exit_code"] = 1
        quality["runner_errors"].append(f"powerbench failed: {exc}")
    finally:
        record["samples"] = sampler.stop()
    record["events"] = events
    by_type: dict[str, list] = {}
    for event in events:
        by_type.setdefault(event.get("type"), []).append(event)
    if len(by_type.get("result", [])) == 1:
        record["benchmark"] = by_type["result"][0]
    else:
        quality["runner_errors"].append("Benchmark did not emit exactly one result")
    for kind, key in (("treatment_protocol", "treatment_protocol"), ("active_reference_result", "active_reference")):
        if len(by_type.get(kind, [])) == 1:
            record[key] = by_type[kind][0]
    devices = by_type.get("device", [])
    if len(devices) == 1:
        record["cuda_device"] = devices[0]
        if devices[0].get("uuid") != device.uuid:
            quality["runner_errors"].append("Actual benchmark CUDA UUID did not match selected physical NVML GPU")
    try:
        record["phases"] = phase_records(events, record["samples"])
    except ValueError as exc:
        quality["runner_errors"].append(f"Invalid benchmark phases: {exc}")
    bench = record["benchmark"]
    for key in ("workload", "access", "blocks", "threads", "iterations_per_launch"):
        if key in bench and key not in record["config"]:
            record["config"][key] = bench[key]
    record["workload"] = bench.get("workload")
    record["status"] = "complete" if not quality["runner_errors"] else "failed"
    quality["valid"] = not quality["runner_errors"]
    return record
