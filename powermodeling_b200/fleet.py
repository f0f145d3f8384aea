"""One workload arm on every GPU of a node at once, one process per GPU.

The reference runs a plan's arms per CUDA device (powermodeling/runner.py:483,
``run_plan`` with one device and one clock context each, clocks.py:92).  Here
``gpu_arm`` runs one powerbench arm on one CUDA device from the calling
process, with that GPU's own native NVML sampler bound to its UUID; with
``capture=True`` the arm is a captured trial (idle, measure, idle phases)
analysed on that GPU, so each GPU reports its own energy per unit of work.
``run_fleet`` starts one process per GPU (spawned, so no CUDA context is
inherited), releases them together and collects per-GPU rows; the fleet
rate is the sum of the per-GPU rates, and every row carries the clocks and
power its GPU ran at.  Clocks are left as the GPUs have them (changing them
is the runner's clock policy, not this module's).

``python -m powermodeling_b200.fleet --gpus N [--capture] -- <powerbench args>``
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import statistics
import sys
import time
from typing import Any

RATE_KEYS = ("throughput_bytes_s", "throughput_ops_s", "throughput_elements_s", "throughput_sfu_instructions_s")
ENERGY_KEYS = ("board_power_w", "idle_power_w", "pj_per_logical_byte", "total_pj_per_logical_byte", "total_pj_per_flop",
               "operational_idle_increment_pj_per_flop", "sfu_reference_delta_pj_per_instruction", "total_pj_per_element",
               "sm_clock_mhz", "memory_clock_mhz", "valid")


def _describe(index: int) -> dict:
    from . import powerbench
    return next(r for r in powerbench.run(["--describe", "--device", str(index)]) if r["type"] == "device")


def gpu_arm(index: int, args: list, capture: bool = False, interval_s: float = 0.02) -> dict[str, Any]:
    """Arm ``args`` on CUDA device ``index`` from this process, sampled by that GPU's NVML handle."""
    from . import powerbench
    from .telemetry import NvmlDevice, Sampler
    dev = _describe(index)
    device = NvmlDevice(uuid=dev["uuid"])
    row: dict[str, Any] = {"device": index, "uuid": dev["uuid"], "name": dev.get("name")}
    try:
        argv = [*map(str, args), "--device", str(index)]
        if capture:
            from .analysis import analyze_trial
            from .capture import capture_trial
            record = capture_trial(argv, device, sample_interval_s=0.01)
            result = record["benchmark"]
            trial = analyze_trial(record)
            row.update({k: trial.get(k) for k in ENERGY_KEYS}, issues=trial.get("issues"))
        else:
            sampler = Sampler(device, interval_s=interval_s).start()
            try:
                records = powerbench.run(argv)
            finally:
                samples = sampler.stop()
            result = next(r for r in records if r["type"] == "result")
            busy = [s for s in samples if s.get("sm_clock_mhz")]
            for key, field in (("sm_mhz", "sm_clock_mhz"), ("mem_mhz", "memory_clock_mhz"), ("power_w", "power_w")):
                values = [s[field] for s in busy if s.get(field) is not None]
                row[key] = statistics.median(values) if values else None
            row["clock_event_reasons"] = sorted({n for s in busy for n in (s.get("throttle_reason_names") or [])})
    finally:
        device.close()
    row.update({k: result.get(k) for k in RATE_KEYS if result.get(k) is not None},
               duration_s=result.get("duration_s"), checksum=result.get("checksum"))
    return row


def _worker(index: int, args: list, capture: bool, start, out) -> None:
    try:
        _describe(index)                 # context and library up before the common start
        start.wait(timeout=300)
        out.put((index, gpu_arm(index, args, capture)))
    except BaseException as exc:        # reported to the parent, which raises
        out.put((index, {"device": index, "error": f"{type(exc).__name__}: {exc}"}))


def run_fleet(args: list, gpus: int, capture: bool = False, timeout_s: float = 900.0) -> dict[str, Any]:
    """``args`` on GPUs 0..gpus-1 at once; per-GPU rows and the summed rates."""
    ctx = mp.get_context("spawn")
    start, out = ctx.Barrier(gpus + 1), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(i, list(args), capture, start, out)) for i in range(gpus)]
    for p in procs:
        p.start()
    start.wait(timeout=300)
    t0 = time.time()
    rows = {}
    try:
        for _ in range(gpus):
            index, row = out.get(timeout=timeout_s)
            rows[index] = row
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    failed = [r for r in rows.values() if "error" in r]
    if failed:
        raise RuntimeError(f"fleet arm failed on {len(failed)} GPU(s): {failed[0]['error']}")
    return fleet_summary([rows[i] for i in sorted(rows)], wall_s=time.time() - t0)


def fleet_summary(rows: list[dict], wall_s: float | None = None) -> dict[str, Any]:
    """Sum of each rate over the GPUs, with the per-GPU spread."""
    out: dict[str, Any] = {"gpus": len(rows), "per_gpu": rows, "wall_s": wall_s}
    for key in RATE_KEYS:
        values = [r[key] for r in rows if r.get(key) is not None]
        if values:
            out[key] = {"sum": sum(values), "min": min(values), "max": max(values)}
    return out


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--" not in argv:
        sys.exit("usage: python -m powermodeling_b200.fleet --gpus N [--capture] -- <powerbench args>")
    split = argv.index("--")
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, required=True)
    parser.add_argument("--capture", action="store_true", help="captured trials analysed for energy per unit of work")
    a = parser.parse_args(argv[:split])
    print(json.dumps(run_fleet(argv[split + 1:], a.gpus, a.capture), default=str))
    return 0


if __name__ == "__main__":
    sys.exit(main())
