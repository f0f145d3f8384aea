"""Seeded synthetic sweeps shaped like the runner's trial records.

The analysis workload is a sweep of ``points`` conditions, each measured
``repeats`` times.  One repeat is a paired trial in the layout that
``powermodeling.runner.capture_trial`` writes (runner.py:301-328, 398-480):
``idle_pre`` -> two active arms (treatment ``measure`` and the integer
``active_reference``) in AB or BA order by repeat parity (planner.py:624-633)
-> ``idle_post``.  Telemetry is one global host stream sampled every
``interval_s`` plus U(0, jitter) on monotone int64 nanosecond stamps; each
phase keeps the samples inside its window plus one neighbour on each side,
as runner.py:177-205 slices them.  Epochs are whole seconds placed strictly
inside sample coverage.

No field here is a measurement of hardware: the power levels are draws from
the stated normal distributions and the record says so in ``device.name``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

ANALYSIS_POLICY = {"trim_s": 0.0, "idle_trim_s": 0.0, "min_measure_s": 1.0, "min_idle_s": 0.5}
"""Policy under which 3 s arms and 1 s idles qualify (defaults need 5 s / 4 s)."""


@dataclass(frozen=True)
class SweepShape:
    points: int = 64
    repeats: int = 4
    arm_s: float = 3.0
    idle_s: float = 1.0
    interval_s: float = 0.010
    jitter_s: float = 0.002
    active_w: tuple = (450.0, 15.0)
    idle_w: tuple = (90.0, 3.0)
    reference_w: tuple = (300.0, 10.0)
    ops_range: tuple = (1e12, 1e13)
    epochs_per_arm: int = 3
    with_energy_counter: bool = False
    workload: str = "tensor"


def _arm_epochs(start_ns, end_ns, count, ops_total, bytes_total):
    """``count`` equal epochs spanning [start+5 ms, end-5 ms] of the arm."""
    lo, hi = start_ns + 5_000_000, end_ns - 5_000_000
    cuts = np.linspace(lo, hi, count + 1).astype(np.int64)
    out = []
    for i in range(count):
        a, b = int(cuts[i]), int(cuts[i + 1])
        out.append({"host_monotonic_start_ns": a, "host_monotonic_end_ns": b,
                    "start_s": a / 1e9, "end_s": b / 1e9, "batches": 1,
                    "operations": ops_total / count, "logical_bytes": bytes_total / count,
                    "counts_exact": True, "counter_readback_ns": 0})
    return out


def make_trial(rng: np.random.Generator, shape: SweepShape, point: int, repeat: int, ops: float,
               uuid: str = "GPU-00000000-0000-0000-0000-0000000000b2", pid: int = 4242) -> dict:
    """One paired trial record; ``rng`` drives every random draw, ``ops`` is the point's count."""
    order = "AB" if repeat % 2 == 0 else "BA"
    t0 = 1_000_000_000_000 + point * 100_000_000_000 + repeat * 20_000_000_000
    idle_ns, arm_ns = int(shape.idle_s * 1e9), int(shape.arm_s * 1e9)
    arms = ["idle_pre"] + (["active_reference", "measure"] if order == "AB" else ["measure", "active_reference"]) + ["idle_post"]
    bounds, cursor = {}, t0 + 20_000_000
    for name in arms:
        length = idle_ns if name.startswith("idle") else arm_ns
        bounds[name] = (cursor, cursor + length)
        cursor += length + (3_000_000 if not name.startswith("idle") else 1_000_000)
    stream_end = cursor + 20_000_000
    # Global monotone sample clock: 10 ms ticks plus U(0, 2 ms) jitter.
    ticks = np.arange(t0, stream_end, int(shape.interval_s * 1e9), dtype=np.int64)
    jitter = rng.integers(0, int(shape.jitter_s * 1e9) + 1, size=ticks.size, dtype=np.int64)
    stamps = ticks + jitter
    power = np.empty(stamps.size)
    phase_of = np.full(stamps.size, -1)
    levels = {"idle_pre": shape.idle_w, "idle_post": shape.idle_w,
              "measure": shape.active_w, "active_reference": shape.reference_w}
    for k, name in enumerate(arms):
        a, b = bounds[name]
        phase_of[(stamps >= a) & (stamps <= b)] = k
    for k, name in enumerate(arms):
        mask = phase_of == k
        mu, sd = levels[name]
        power[mask] = rng.normal(mu, sd, size=int(mask.sum()))
    gaps = phase_of == -1
    power[gaps] = rng.normal(shape.idle_w[0], shape.idle_w[1], size=int(gaps.sum()))
    energy = None
    if shape.with_energy_counter:
        dt = np.diff(stamps, prepend=stamps[0]) / 1e9
        energy = (np.int64(7_000_000_000) + np.cumsum(np.rint(power * dt * 1000.0)).astype(np.int64))
    active = (phase_of >= 0) & np.isin(phase_of, [arms.index("measure"), arms.index("active_reference")])
    samples = []
    for i in range(stamps.size):
        s = {"t_s": int(stamps[i]) / 1e9, "power_w": float(power[i]),
             "graphics_clock_mhz": 1965, "sm_clock_mhz": 1965, "memory_clock_mhz": 3996,
             "temperature_c": 55, "throttle_reasons": 0, "power_limit_w": 1000.0,
             "enforced_power_limit_w": 1000.0, "pstate": 0,
             "compute_processes": [{"pid": pid, "used_gpu_memory_bytes": None}] if active[i] else [],
             "graphics_processes": []}
        if energy is not None:
            s["energy_mj"] = int(energy[i])
        samples.append(s)
    phases = {}
    for name in arms:
        a, b = bounds[name]
        inside = np.nonzero((stamps >= a) & (stamps <= b))[0]
        lo, hi = max(0, int(inside[0]) - 1), min(stamps.size, int(inside[-1]) + 2)
        phases[name] = {"start_s": a / 1e9, "end_s": b / 1e9, "samples": samples[lo:hi]}
    m0, m1 = bounds["measure"]
    r0, r1 = bounds["active_reference"]
    geometry = {"blocks": 296, "threads": 256, "batch_launches": 16, "iterations_per_launch": 1024}
    benchmark = {"workload": shape.workload, "duration_s": (m1 - m0) / 1e9, "host_duration_s": (m1 - m0) / 1e9,
                 "operations": ops, "logical_bytes": 0.0,
                 "measure_epochs": _arm_epochs(m0, m1, shape.epochs_per_arm, ops, 0.0),
                 "paired_reference_context_allocated": True,
                 "sanity": {"finite_output_sample": True, "requested_sm_coverage_complete": True},
                 **geometry}
    reference = {"workload": "control", "reference_kind": "issue_loop", "duration_s": (r1 - r0) / 1e9,
                 "host_duration_s": (r1 - r0) / 1e9, "operations": 0, "logical_bytes": 0,
                 "measure_epochs": _arm_epochs(r0, r1, shape.epochs_per_arm, 0.0, 0.0),
                 "sanity": {"requested_sm_coverage_complete": True}, **geometry}
    protocol = {"kind": "paired_active_reference", "order": order, "same_process": True,
                "same_allocations": True, "same_clock_policy": True, "launch_geometry_matched": True,
                "paired_reference_context_allocated": True, "reference_workload": "control",
                "reference_kind": "issue_loop"}
    return {"schema_version": 1, "trial_id": f"p{point:05d}-r{repeat}", "condition_id": f"p{point:05d}",
            "repeat": repeat, "workload": shape.workload, "status": "complete",
            "config": {"gpu_uuid": uuid, "graphics_clock_mhz": 1965, "memory_clock_mhz": 3996,
                       "blocks": 296, "threads": 256, "point": point, "repeat": repeat},
            "benchmark": benchmark, "active_reference": reference, "treatment_protocol": protocol,
            "phases": phases, "device": {"name": "Synthetic sweep trace, not measured hardware",
                                         "uuid": uuid, "power_limit_w": 1000.0},
            "quality": {"valid": True, "measurement_pid": pid}}


def make_sweep(shape: SweepShape = SweepShape(), seed: int = 0, first_point: int = 0) -> list[dict]:
    """``shape.points * shape.repeats`` trial records from one seeded generator.

    Points are numbered from ``first_point``, so sweeps built for different
    shards of a larger sweep never share a group key.
    """
    rng = np.random.default_rng(seed)
    ops = rng.uniform(*shape.ops_range, size=shape.points)
    return [make_trial(rng, shape, first_point + p, r, float(ops[p]))
            for p in range(shape.points) for r in range(shape.repeats)]
