"""Workload-arm measurements on one GPU: the benchmark configurations' grids through powerbench.

Each function runs the powerbench engine in this process over one
configuration's grid and returns one row per point:

* ``hbm_sweep`` - streaming reads and copies (16-byte and 4-byte accesses,
  .cg/.cs/.ca): working set 256 MiB-16 GiB, grid 148 x {1,2,4,8} x
  {128..1024} threads, stride 1-32, base offset 0-124 bytes, random_word and
  LCG payloads; logical bytes/s against the interface ceiling from the
  sampled memory clock x bus width (cuda/gpu_bench.cu:326-406, 659-668;
  powermodeling/hbm_bandwidth.py:12).
* ``cache_sweep`` - L1 .ca re-reads of 16-192 KiB per SM (one CTA per SM) and
  the dependent chase over 4-96 MiB, one warp per SM on every SM, 1e6 loads
  each, as u32 word links (the reference's permutation) and as u64 links on
  128-byte lines; per-SM cycles per access (gpu_bench.cu:457-473, 722-737).
* ``sfu_sweep`` - EX2, LG2, RCP, RSQRT, SQRT and tanh.approx at grids of
  148 x k CTAs (k = 1..8) x 256 threads, 4 chains, with the matched
  register-loop control (sfu.cuh:43-105): MUFU ops per SM per clock.
* ``energy_arm`` - one trial captured under the NVML sampler
  (capture.capture_trial) and analysed by the GPU analysis: pJ per logical
  byte, per FLOP or, with the paired control, the differential pJ per SFU
  instruction (powermodeling/analysis.py:713-762, 937-946).

``python -m powermodeling_b200.sweeps --out FILE`` runs every grid and
writes the rows as JSON.  Clocks are left as the GPU has them.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
import time
from typing import Any

from . import powerbench

SFU_OPCODES = ("ex2", "lg2", "rcp", "rsqrt", "sqrt", "tanh")
# A measurement window of a few fixed batches (the engine times them with CUDA events).
QUICK = ["--seconds", "1", "--warmup-seconds", "0", "--idle-seconds", "0", "--warmup-batches", "1"]


def _result(args: list) -> tuple[dict, dict]:
    records = powerbench.run([str(a) for a in args])
    device = next(r for r in records if r["type"] == "device")
    return device, next(r for r in records if r["type"] == "result")


def describe() -> dict:
    return next(r for r in powerbench.run(["--describe"]) if r["type"] == "device")


def _clock_sampler(uuid: str):
    """A native NVML sampler at 20 ms (SM and memory clocks during a point), or None without NVML."""
    try:
        from .telemetry import NvmlDevice, Sampler
        device = NvmlDevice(uuid=uuid)
        return device, Sampler(device, interval_s=0.02).start()
    except Exception:                                     # no NVML: rows carry no clock
        return None


def _clock_stop(handle) -> dict:
    if handle is None:
        return {}
    device, sampler = handle
    try:
        samples = sampler.stop()
    finally:
        device.close()
    sm = [s["sm_clock_mhz"] for s in samples if s.get("sm_clock_mhz")]
    mem = [s["memory_clock_mhz"] for s in samples if s.get("memory_clock_mhz")]
    return {"sm_mhz": statistics.median(sm) if sm else None, "mem_mhz": statistics.median(mem) if mem else None}


# ---------------------------------------------------------------------------- HBM
def _hbm_args(sms: int, *, ws: int, blocks_per_sm: int = 8, threads: int = 256, stride: int = 1, offset: int = 0,
              policy: str = "cs", vector: bool = True, access: str = "read", fill: str = "random_word") -> list:
    """The geometry of one HBM point: every launch covers the working set once."""
    unit = 16 if vector else 4
    lanes = sms * blocks_per_sm * threads
    iterations = max(1, ws // (unit * lanes))
    args = ["--workload", "hbm", "--access", access, "--blocks", sms * blocks_per_sm, "--threads", threads,
            "--working-set-bytes", ws, "--iterations", iterations, "--stride-words", stride, "--offset-bytes", offset,
            "--batch-launches", 4, "--fill", fill]
    if access == "read":
        args += ["--read-cache-policy", policy]
    if vector:
        args += ["--memory-vector-bytes", 16]
    return args


def _hbm_point(sms: int, batches: int = 3, **point) -> list:
    return _hbm_args(sms, **point) + ["--fixed-batches", batches, *QUICK]


def hbm_points(sms: int, quick: bool = False) -> list[tuple[str, dict]]:
    """(factor, point) pairs: one factor at a time around 4 GiB, 148 x 8 x 256, stride 1, offset 0, 16-byte .cs reads."""
    base = {"ws": 4 << 30}
    pts: list[tuple[str, dict]] = [("base", dict(base))]
    if quick:
        return pts + [("access", dict(base, access="copy")), ("scalar", dict(base, vector=False, policy="cg")),
                      ("fill", dict(base, fill="lcg"))]
    for e in range(28, 35):
        pts.append(("working_set", {"ws": 1 << e}))
        pts.append(("working_set_copy", {"ws": 1 << e, "access": "copy"}))
    for bps in (1, 2, 4, 8):
        for threads in (128, 256, 512, 1024):
            pts.append(("grid", dict(base, blocks_per_sm=bps, threads=threads)))
    for stride in (1, 2, 4, 8, 16, 32):
        pts.append(("stride_scalar_cg", dict(base, vector=False, policy="cg", stride=stride)))
        pts.append(("stride_vector_cs", dict(base, stride=stride)))
    for offset in range(0, 128, 4):
        pts.append(("offset_scalar_cg", dict(base, vector=False, policy="cg", offset=offset)))
    for offset in range(0, 128, 16):
        pts.append(("offset_vector_cs", dict(base, offset=offset)))
    for policy in ("cg", "cs", "ca"):
        pts.append(("policy_vector", dict(base, policy=policy)))
        pts.append(("policy_scalar", dict(base, policy=policy, vector=False)))
    pts.append(("fill_lcg", dict(base, fill="lcg")))
    pts.append(("fill_lcg_copy", dict(base, fill="lcg", access="copy")))
    return pts


def hbm_sweep(sms: int, quick: bool = False) -> list[dict]:
    rows = []
    for factor, point in hbm_points(sms, quick):
        device, r = _result(_hbm_point(sms, **point))
        rows.append({"factor": factor, **point, "gbs": r["throughput_bytes_s"] / 1e9, "bytes": r["logical_bytes"],
                     "duration_s": r["duration_s"], "validation": (r.get("memory_read_validation") or {}).get("status"),
                     "bus_bits": device["memory_bus_width_bits"]})
    return rows


def with_theory(rows: list[dict], mem_mhz: float) -> list[dict]:
    """Adds the interface ceiling 2 x memory MHz x 1e6 x bus bits / 8 and each row's fraction of it."""
    for row in rows:
        theory = 2 * mem_mhz * 1e6 * row["bus_bits"] / 8 / 1e9
        row["theory_gbs"] = theory
        row["frac_of_theory"] = row["gbs"] / theory
    return rows


# ---------------------------------------------------------------------------- caches
def cache_sweep(sms: int, quick: bool = False, loads: int = 1_000_000) -> dict[str, list[dict]]:
    l1, chase = [], []
    for kib in ((192,) if quick else (16, 32, 64, 96, 128, 192)):
        ws = sms * kib * 1024
        threads = 256
        iterations = 4096
        _, r = _result(["--workload", "l1", "--blocks", sms, "--threads", threads, "--working-set-bytes", ws,
                        "--iterations", iterations, "--batch-launches", 4, "--fixed-batches", 3, *QUICK])
        l1.append({"kib_per_sm": kib, "gbs": r["throughput_bytes_s"] / 1e9,
                   "validation": (r.get("memory_read_validation") or {}).get("status")})
    for granularity in ("line", "word"):
        for mib in ((96,) if quick else (4, 8, 16, 32, 64, 96)):
            args = ["--workload", "l2_latency", "--chase-granularity", granularity, "--blocks", sms, "--threads", 32,
                    "--working-set-bytes", mib << 20, "--iterations", loads, "--batch-launches", 1, "--fixed-batches", 1,
                    *QUICK]
            _, r = _result(args)
            per_sm = [v["cycles_per_access"] for v in r["latency_probe"]["per_sm"].values() if v["loads"]]
            chase.append({"granularity": granularity, "mib": mib, "sms": len(per_sm), "loads_per_sm": loads,
                          "cycles_per_access_median": statistics.median(per_sm) if per_sm else None,
                          "cycles_per_access_min": min(per_sm, default=None),
                          "cycles_per_access_max": max(per_sm, default=None), "checksum": r["checksum"]})
    return {"l1": l1, "chase": chase}


# ---------------------------------------------------------------------------- SFU
def sfu_sweep(sms: int, ks=range(1, 9), opcodes=SFU_OPCODES, iterations: int = 1 << 20,
              uniform_input: bool = False) -> list[dict]:
    """MUFU throughput of each opcode and of the matched control at 148 x k CTAs of 256 threads."""
    rows = []
    for op in opcodes:
        for k in ks:
            blocks = sms * k
            args = ["--workload", "sfu_" + op, "--grid-mode", "fixed", "--blocks", blocks, "--threads", 256,
                    "--sfu-lanes", blocks * 256, "--sfu-chains", 4, "--iterations", iterations, "--batch-launches", 1,
                    "--fixed-batches", 2, *QUICK]
            if uniform_input:
                args += ["--sfu-input", "uniform_0p5_2"]
            handle = _clock_sampler(describe()["uuid"]) if k in (1, 8) else None
            _, r = _result(args)
            clock = _clock_stop(handle)
            row = {"opcode": op, "k": k, "blocks": blocks, "ops_s": r["throughput_ops_s"], "checksum": r["checksum"],
                   "validation_passed": r["sanity"]["numerical_validation_passed"], **clock}
            if uniform_input:
                row["thread_xor_checksum"] = r.get("sfu_thread_xor_checksum")
            rows.append(row)
    return rows


def per_sm_clock(rows: list[dict], sms: int, sm_mhz: float) -> list[dict]:
    """MUFU ops per SM per clock, at each row's sampled SM clock when it has one."""
    for row in rows:
        mhz = row.get("sm_mhz") or sm_mhz
        row["ops_per_sm_per_clock"] = row["ops_s"] / (sms * mhz * 1e6)
    return rows


# ---------------------------------------------------------------------------- energy
ENERGY_KEYS = ("board_power_w", "idle_power_w", "incremental_power_w", "throughput_ops_s", "throughput_bytes_s",
               "pj_per_logical_byte", "total_pj_per_logical_byte", "total_pj_per_flop",
               "operational_idle_increment_pj_per_flop", "operational_idle_increment_pj_per_logical_bit",
               "total_pj_per_logical_bit", "sfu_reference_delta_pj_per_instruction", "sfu_reference_delta_power_w",
               "total_pj_per_instruction", "throughput_sfu_instructions_s", "paired_active_reference_power_w",
               "sm_clock_mhz", "memory_clock_mhz", "valid", "paired_active_reference_eligible")


def energy_arm(args: list, seconds: float = 10.0, idle: float = 6.0, warmup: float = 1.0) -> dict[str, Any]:
    """One trial of ``args`` captured under the native sampler (10 ms) and analysed on the GPU with the
    reference's default policy: energy per unit of work over the aligned measure epochs."""
    from .analysis import analyze_trial
    from .capture import capture_trial
    from .telemetry import NvmlDevice
    device = NvmlDevice(uuid=describe()["uuid"])
    try:
        record = capture_trial([*map(str, args), "--seconds", seconds, "--warmup-seconds", warmup,
                                "--idle-seconds", idle], device, sample_interval_s=0.01,
                               trial_id=f"energy-{args[1]}-{int(time.time() * 1e3)}")
    finally:
        device.close()
    trial = analyze_trial(record)
    out = {k: trial.get(k) for k in ENERGY_KEYS}
    out.update(issues=trial.get("issues"), samples=len(record.get("samples", [])),
               measure_s=(trial.get("phases", {}).get("measure") or {}).get("duration_s"))
    return out


def energy_arms(sms: int, sfu: bool = True) -> dict[str, dict]:
    """pJ per logical byte of the 16-byte HBM read, pJ per FLOP of the tcgen05 arm (and of cuBLAS),
    differential pJ per SFU instruction of EX2 against its matched register-loop control."""
    out = {"hbm_read": energy_arm(_hbm_args(sms, ws=4 << 30)),
           "tensor_tcgen05": energy_arm(["--workload", "tensor", "--blocks", sms, "--threads", 128, "--iterations", 8192,
                                         "--tensor-accumulators", 2, "--batch-launches", 4])}
    if sfu:
        out["sfu_ex2_paired"] = energy_arm(["--workload", "sfu_ex2", "--grid-mode", "fixed", "--blocks", sms * 8,
                                            "--threads", 256, "--sfu-lanes", sms * 8 * 256, "--sfu-chains", 4,
                                            "--iterations", 65536, "--batch-launches", 1, "--paired-reference",
                                            "--reference-order", "AB"])
    return out


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--out", required=True)
    parser.add_argument("--quick", action="store_true")
    parser.add_argument("--only", choices=("hbm", "cache", "sfu", "energy"), action="append")
    a = parser.parse_args(argv)
    dev = describe()
    sms = dev["sm_count"]
    parts = a.only or ["hbm", "cache", "sfu", "energy"]
    result: dict[str, Any] = {"device": {k: dev.get(k) for k in ("name", "uuid", "sm_count", "memory_bus_width_bits")}}
    handle = _clock_sampler(dev["uuid"])
    t0 = time.time()
    if "hbm" in parts:
        result["hbm"] = hbm_sweep(sms, a.quick)
    if "cache" in parts:
        result["cache"] = cache_sweep(sms, a.quick)
    if "sfu" in parts:
        result["sfu"] = sfu_sweep(sms, ks=(8,) if a.quick else range(1, 9))
        result["sfu_uniform_input"] = sfu_sweep(sms, ks=(8,), uniform_input=True)
    clock = _clock_stop(handle)
    if "hbm" in result and clock.get("mem_mhz"):
        with_theory(result["hbm"], clock["mem_mhz"])
    for key in ("sfu", "sfu_uniform_input"):
        if key in result:
            per_sm_clock(result[key], sms, clock.get("sm_mhz") or 1965.0)
    if "energy" in parts:
        result["energy"] = energy_arms(sms)
    result["clocks"] = clock
    result["seconds"] = time.time() - t0
    with open(a.out, "w") as f:
        json.dump(result, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
