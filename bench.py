"""Benchmark of the analysis hot path: bootstrap resamples per second.

Workload: 64 sweep points x 4 repeats of paired trials (3 s arms, 1 s idles,
10 ms samples with 0-2 ms jitter, N(450,15)/N(300,10)/N(90,3) W), seed 0 per
rank; one step analyzes every trial (phase integrals over aligned epochs,
idle-delta, paired pJ/FLOP) and computes every group's medians and
10 000-draw percentile-bootstrap intervals.  ``value`` counts
resamples = sum over groups of (metrics with an interval) x B per second of
device time with inputs resident in HBM (L2 flushed between steps); ``e2e``
is the same metric through the host-buffer C-ABI call pm_analyze_sweep.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
Under torchrun each rank analyzes its own sweep (weak scaling); device time
is the maximum over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

RESAMPLES = 10000
POINTS, REPEATS = 64, 4
METRIC = "bootstrap resamples/s"
WORKLOAD = "analysis: 64 points x 4 paired repeats, 3 s arms / 1 s idles at 10 ms, B=10000"


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,clocks.mem")

    def __init__(self, index: int):
        self.index, self.proc, self.path = index, None, None

    def start(self):
        try:
            self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"pmb200_clocks_{os.getpid()}_{id(self)}.csv"
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = [line.split(", ") for line in self.path.read_text().splitlines() if line.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 10 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 10 and r[2].replace(".", "").isdigit()]
        mem = [float(r[9]) for r in rows if len(r) >= 10 and r[9].strip().replace(".", "").isdigit()]
        power = [float(r[3]) for r in rows if len(r) >= 10 and r[3].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({name for r in rows if len(r) >= 10 for name, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "mem_mhz": statistics.median(mem) if mem else None,
                "power_w_median": statistics.median(power) if power else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------- workload
def build_workload(seed: int):
    """Records, packed arrays and group structure (keys/seeds) of one rank's sweep."""
    from powermodeling_b200 import analysis as A
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(points=POINTS, repeats=REPEATS), seed=seed)
    policy = A.AnalysisPolicy(**ANALYSIS_POLICY)
    packed, _, _ = A.prepare(records)
    trials = A.analyze_trials(records, policy)              # one untimed pass for the group keys
    buckets: dict[str, list[int]] = {}
    for i, t in enumerate(trials):
        buckets.setdefault(A.group_key(t), []).append(i)
    keys = sorted(buckets)
    members = [buckets[k] for k in keys]
    seeds = [A.group_seed(k) for k in keys]
    return records, policy, packed, members, seeds


def device_arrays(packed, torch):
    from powermodeling_b200 import _native as N
    dev = {}
    t = N.Trials()
    t.n_trials, t.max_phase_samples, t.n_samples, t.n_epochs = packed.n_trials, packed.max_phase_samples, packed.n_samples, packed.n_epochs
    for name, dtype, _ in N.TRIAL_ARRAYS + N.EPOCH_ARRAYS + N.TAIL_ARRAYS:
        a = packed.arrays[name]
        d = torch.from_numpy(a.copy()).cuda() if a.size else torch.empty(1, dtype=torch.uint8, device="cuda")
        dev[name] = d
        setattr(t, name, d.data_ptr())
    in_bytes = sum(packed.arrays[n].nbytes for n, _, _ in N.TRIAL_ARRAYS + N.EPOCH_ARRAYS + N.TAIL_ARRAYS)
    return t, dev, in_bytes


def run_b200(args, rank: int, world: int) -> dict | None:
    import torch
    import torch.distributed as dist
    from powermodeling_b200 import _native as N

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    lib = N.library()
    records, policy, packed, members, seeds = build_workload(seed=rank)
    n, M, G = packed.n_trials, len(__import__("powermodeling_b200.analysis", fromlist=["METRICS"]).METRICS), len(members)
    trials, keep, in_bytes = device_arrays(packed, torch)
    PO, TO = N.layout("PM_PO_COUNT"), N.layout("PM_TO_COUNT")
    out = {"phase_out": torch.empty(n * 5 * PO, dtype=torch.float64, device="cuda"),
           "phase_flags": torch.empty(n * 5, dtype=torch.int32, device="cuda"),
           "trial_out": torch.empty(n * TO, dtype=torch.float64, device="cuda"),
           "issue_bits": torch.empty(n * 4, dtype=torch.int64, device="cuda"),
           "metrics": torch.empty(n * M, dtype=torch.float64, device="cuda"),
           "valid": torch.empty(n, dtype=torch.uint8, device="cuda")}
    results = N.TrialResults(*(out[k].data_ptr() for k in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid")))
    out_bytes = sum(v.numel() * v.element_size() for v in out.values())
    offsets = np.zeros(G + 1, dtype=np.int32)
    np.cumsum([len(m) for m in members], out=offsets[1:])
    rows = np.concatenate([np.asarray(m, dtype=np.int32) for m in members])
    d_off, d_rows = torch.from_numpy(offsets).cuda(), torch.from_numpy(rows).cuda()
    d_seeds = torch.from_numpy(np.asarray(seeds, dtype=np.uint64).view(np.int64)).cuda()
    med, lo, hi = (torch.empty(G * M, dtype=torch.float64, device="cuda") for _ in range(3))
    job = N.BootstrapJob(G, M, int(rows.size), n, RESAMPLES, max(len(m) for m in members),
                         out["metrics"].data_ptr(), d_off.data_ptr(), d_rows.data_ptr(), out["valid"].data_ptr(),
                         d_seeds.data_ptr(), med.data_ptr(), lo.data_ptr(), hi.data_ptr())
    a_scr = lib.pm_analyze_scratch_bytes(n, packed.max_phase_samples)
    b_scr = lib.pm_bootstrap_scratch_bytes(G, job.max_members, RESAMPLES)
    scratch = torch.empty(max(1, a_scr + b_scr), dtype=torch.uint8, device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    sptr = C.c_void_p(stream.cuda_stream)
    native_policy = policy.native()

    def step():
        N.check(lib.pm_analyze_trials_device(trials, native_policy, results, C.c_void_p(scratch.data_ptr()), a_scr, sptr), "analyze")
        e_mid.record(stream)
        N.check(lib.pm_group_bootstrap_device(job, C.c_void_p(scratch.data_ptr() + a_scr), b_scr, sptr), "bootstrap")

    e0, e_mid, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    resamples_per_step = int(torch.isfinite(lo).sum().item()) * RESAMPLES
    # correctness guard on the timed configuration: every trial valid, every group filled
    assert int(out["valid"].sum().item()) == n, "synthetic trials must all be valid"
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    t_analyze, t_boot = [], []
    for _ in range(args.steps):
        flush.zero_()                                   # L2 flush, outside the timed events
        e0.record(stream)
        step()
        e1.record(stream)
        e1.synchronize()
        t_analyze.append(e0.elapsed_time(e_mid))
        t_boot.append(e_mid.elapsed_time(e1))
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    if world > 1:
        dist.barrier()
    total_ms = sum(t_analyze) + sum(t_boot)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = resamples_per_step * world / (ms_per_step / 1e3)

    # ---- end to end: host buffers through pm_analyze_sweep ----------------------
    from powermodeling_b200.pack import trials_struct
    host_trials = trials_struct(packed)
    h_out = {"phase_out": np.empty(n * 5 * PO), "phase_flags": np.empty(n * 5, dtype=np.uint32),
             "trial_out": np.empty(n * TO), "issue_bits": np.empty(n * 4, dtype=np.uint64),
             "metrics": np.empty(n * M), "valid": np.empty(n, dtype=np.uint8)}
    h_results = N.TrialResults(*(h_out[k].ctypes.data for k in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid")))
    h_med, h_lo, h_hi = (np.empty(G * M) for _ in range(3))
    seeds_np = np.asarray(seeds, dtype=np.uint64)
    h_job = N.BootstrapJob(G, M, int(rows.size), n, RESAMPLES, 0, None, offsets.ctypes.data, rows.ctypes.data, None,
                           seeds_np.ctypes.data, h_med.ctypes.data, h_lo.ctypes.data, h_hi.ctypes.data)
    for _ in range(args.warmup):
        N.check(lib.pm_analyze_sweep(host_trials, native_policy, h_results, h_job), "pm_analyze_sweep")
    if world > 1:
        dist.barrier()
    e2e_times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        N.check(lib.pm_analyze_sweep(host_trials, native_policy, h_results, h_job), "pm_analyze_sweep")
        e2e_times.append(time.perf_counter() - t0)
    e2e_s = sum(e2e_times) / args.steps
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    assert np.array_equal(np.nan_to_num(h_lo), np.nan_to_num(lo.cpu().numpy())), "e2e and device paths disagree"
    h2d = in_bytes + offsets.nbytes + rows.nbytes + seeds_np.nbytes
    d2h = sum(a.nbytes for a in h_out.values()) + 3 * h_med.nbytes
    if rank != 0:
        return None
    peaks = measured_peaks()
    a_ms, b_ms = statistics.mean(t_analyze), statistics.mean(t_boot)
    dominant = "bootstrap_kernel" if b_ms >= a_ms else "analyze_kernel"
    roofline = roofline_entry(dominant, a_ms, b_ms, in_bytes, out_bytes, G, M, packed, peaks, resamples_per_step)
    line = {"metric": METRIC, "value": value, "unit": "resamples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "points": POINTS, "repeats": REPEATS, "trials": n, "groups": G,
                       "resamples": RESAMPLES, "samples": packed.n_samples, "l2": "flushed (256 MiB write) between steps",
                       "parallelism": f"sweep-per-gpu x{world}"},
            "e2e": {"value": resamples_per_step * world / e2e_s, "unit": "resamples/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_s * 1e3},
            "gpu_launches": 2 * args.steps,
            "kernels": {"analyze_kernel_ms": a_ms, "bootstrap_kernel_ms": b_ms},
            "roofline": roofline, "clocks": clock_info}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(records, policy)
    if not args.no_arms and world == 1:
        line["arms"] = run_arms(local, peaks)
    return line


# --------------------------------------------------------------------------- workload arms
ARM_QUICK = ["--seconds", "5", "--warmup-seconds", "0", "--idle-seconds", "0", "--warmup-batches", "2"]


def _arm(args):
    from powermodeling_b200 import powerbench
    records = powerbench.run(args)
    device = next(r for r in records if r["type"] == "device")
    return device, next(r for r in records if r["type"] == "result")


def _pynvml_sample_cost(uuid: str, reads: int = 200) -> float | None:
    """Median seconds of one sample read the reference's way: its NVML calls
    (powermodeling/telemetry.py:195-243) from Python through pynvml."""
    try:
        import pynvml as nv
    except ImportError:
        return None
    nv.nvmlInit()
    try:
        h = nv.nvmlDeviceGetHandleByUUID(uuid)
        fields = [(nv.NVML_FI_DEV_POWER_INSTANT, nv.NVML_POWER_SCOPE_GPU),
                  (nv.NVML_FI_DEV_POWER_AVERAGE, nv.NVML_POWER_SCOPE_GPU),
                  (nv.NVML_FI_DEV_POWER_INSTANT, nv.NVML_POWER_SCOPE_MEMORY),
                  (nv.NVML_FI_DEV_POWER_AVERAGE, nv.NVML_POWER_SCOPE_MEMORY)]
        calls = [lambda: nv.nvmlDeviceGetPowerUsage(h), lambda: nv.nvmlDeviceGetFieldValues(h, fields),
                 lambda: nv.nvmlDeviceGetTotalEnergyConsumption(h),
                 lambda: nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_GRAPHICS),
                 lambda: nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                 lambda: nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_MEM),
                 lambda: nv.nvmlDeviceGetTemperature(h, nv.NVML_TEMPERATURE_GPU),
                 lambda: nv.nvmlDeviceGetPerformanceState(h), lambda: nv.nvmlDeviceGetCurrentClocksEventReasons(h),
                 lambda: nv.nvmlDeviceGetUtilizationRates(h), lambda: nv.nvmlDeviceGetPowerManagementLimit(h),
                 lambda: nv.nvmlDeviceGetEnforcedPowerLimit(h), lambda: nv.nvmlDeviceGetComputeRunningProcesses(h),
                 lambda: nv.nvmlDeviceGetGraphicsRunningProcesses(h),
                 lambda: nv.nvmlDeviceGetMPSComputeRunningProcesses(h)]
        times = []
        for _ in range(reads):
            t0 = time.perf_counter()
            for call in calls:
                try:
                    call()
                except nv.NVMLError:
                    pass
            times.append(time.perf_counter() - t0)
        return statistics.median(times)
    finally:
        nv.nvmlShutdown()


def run_telemetry_arm(uuid: str) -> dict:
    """Native sampler: achieved tick rate and query latency at 10 ms and 1 ms intervals."""
    from powermodeling_b200.telemetry import NvmlDevice, Sampler
    out = {}
    device = NvmlDevice(uuid=uuid)
    try:
        for interval in (0.01, 0.001):
            sampler = Sampler(device, interval_s=interval).start()
            time.sleep(1.0)
            samples = sampler.stop()
            q = sorted(s["query_duration_s"] for s in samples)
            span = samples[-1]["t_s"] - samples[0]["t_s"]
            out[f"interval_{interval * 1e3:g}ms"] = {
                "samples": len(samples), "samples_per_s": (len(samples) - 1) / span if span > 0 else None,
                "query_ms_p50": 1e3 * q[len(q) // 2], "query_ms_p99": 1e3 * q[min(len(q) - 1, int(len(q) * 0.99))],
                "fatal": sum(1 for s in samples if s["fatal_errors"])}
    finally:
        device.close()
    cost = _pynvml_sample_cost(uuid)
    out["pynvml_reference_calls_query_ms_p50"] = None if cost is None else 1e3 * cost
    return out


def run_arms(local: int, peaks: dict) -> dict:
    """HBM read/copy, tcgen05 tensor, cuBLAS GEMM and SFU arms through the powerbench engine."""
    sms = 148
    out = {}
    clocks = ClockSampler(local)
    clocks.start()
    hbm = ["--workload", "hbm", "--memory-vector-bytes", "16", "--read-cache-policy", "cs", "--blocks", str(sms * 8),
           "--threads", "256", "--working-set-bytes", str(4 << 30), "--iterations", "1024",
           "--batch-launches", "8", "--fixed-batches", "6", *ARM_QUICK]
    device, r = _arm(hbm)
    sms = device["sm_count"]
    bus = device["memory_bus_width_bits"]
    out["hbm_read"] = {"gbs": r["throughput_bytes_s"] / 1e9, "bytes": r["logical_bytes"], "duration_s": r["duration_s"],
                       "validation": r["memory_read_validation"]["status"], "config": "16 B loads (.cs), 4 GiB, grid 148x8x256"}
    _, r = _arm(["--workload", "hbm", "--access", "copy", "--memory-vector-bytes", "16", "--blocks", str(sms * 8),
                 "--threads", "256", "--working-set-bytes", str(4 << 30), "--iterations", "512", "--batch-launches", "8",
                 "--fixed-batches", "6", *ARM_QUICK])
    out["hbm_copy"] = {"gbs": r["throughput_bytes_s"] / 1e9, "config": "16 B load+store, 4 GiB, grid 148x8x256"}
    tensor = {}
    for acc in (1, 2, 4, 8):
        # 2 s per arm: long enough for the power-capped clock to settle and be sampled.
        arm_clock = ClockSampler(local)
        arm_clock.start()
        _, r = _arm(["--workload", "tensor", "--blocks", str(sms), "--threads", "128", "--iterations", "8192",
                     "--tensor-accumulators", str(acc), "--batch-launches", "4", "--seconds", "2",
                     "--warmup-seconds", "0", "--idle-seconds", "0", "--warmup-batches", "2"])
        c = arm_clock.stop()
        tflops = r["throughput_ops_s"] / 1e12
        entry = {"tflops": tflops, "tile_n": r["tensor_tile_n"], "timeouts": r["tensor_status"]["bounded_wait_timeouts"],
                 "sm_mhz": c.get("sm_mhz"), "power_w": c.get("power_w_median"), "reasons": c.get("reasons")}
        if c.get("sm_mhz"):
            entry["frac_of_dense_peak_at_arm_clock"] = tflops / (8192 * sms * c["sm_mhz"] * 1e6 / 1e12)
        tensor[str(acc)] = entry
    out["tensor_tcgen05"] = tensor
    _, r = _arm(["--workload", "gemm", "--gemm-m", "8192", "--gemm-n", "8192", "--gemm-k", "8192", "--batch-launches", "4",
                 "--fixed-batches", "3", *ARM_QUICK])
    out["gemm_cublas_8192"] = {"tflops": r["throughput_ops_s"] / 1e12}
    _, r = _arm(["--workload", "sfu_ex2", "--grid-mode", "fixed", "--blocks", str(sms * 8), "--threads", "256",
                 "--sfu-lanes", str(sms * 8 * 256), "--sfu-chains", "4", "--iterations", "65536", "--batch-launches", "1",
                 "--fixed-batches", "4", *ARM_QUICK])
    out["sfu_ex2"] = {"ops_s": r["throughput_ops_s"], "checksum": r["checksum"]}
    clock = clocks.stop()
    out["telemetry"] = run_telemetry_arm(device["uuid"])
    mem_mhz = clock.get("mem_mhz") or device["nominal_max_memory_clock_khz"] / 1e3
    theory = 2 * mem_mhz * 1e6 * bus / 8 / 1e9
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    for key in ("hbm_read", "hbm_copy"):
        out[key]["frac_of_measured_copy_peak"] = out[key]["gbs"] / hbm_peak
        out[key]["frac_of_clock_bus_theory"] = out[key]["gbs"] / theory
    out["hbm_theory_gbs"] = theory
    sm_mhz = clock.get("sm_mhz") or 1965.0
    dense_peak = 8192 * sms * sm_mhz * 1e6 / 1e12
    best = max(v["tflops"] for v in tensor.values())
    out["tensor_peak_at_clock_tflops"] = dense_peak
    out["tensor_best_frac_of_dense_clock_peak"] = best / dense_peak
    out["tensor_best_frac_of_measured_bf16_gemm"] = best / peaks.get("bf16_tflops", 1590.0)
    out["sfu_ex2"]["ops_per_sm_per_clock"] = out["sfu_ex2"]["ops_s"] / (sms * sm_mhz * 1e6)
    out["clocks"] = clock
    return out


# DRAM bytes (read + write) per launch from one ncu capture of the same
# workload (profiles/analysis_sweep_64x4_B10000.md); None where none was taken.
NCU_TRAFFIC_BYTES = {"analyze_kernel": 19_193_856, "bootstrap_kernel": None}


def roofline_entry(dominant, a_ms, b_ms, in_bytes, out_bytes, G, M, packed, peaks, resamples):
    hbm = peaks.get("hbm_gbs", 6650.0)
    src = "measured" if not peaks.get("fallback") else "fallback"
    if dominant == "analyze_kernel":
        achieved = (in_bytes + out_bytes) / (a_ms / 1e3) / 1e9
        return {"kernel": dominant, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": NCU_TRAFFIC_BYTES["analyze_kernel"], "peak_source": src,
                "algorithmic_bytes": in_bytes + out_bytes}
    # The bootstrap kernel moves a few KB; its bound is the MT19937 stream (2 words per draw).
    words = 2 * 4 * RESAMPLES * G
    achieved = words * 4 / (b_ms / 1e3) / 1e9
    return {"kernel": dominant, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "traffic": NCU_TRAFFIC_BYTES["bootstrap_kernel"], "peak_source": src,
            "note": "random-stream bytes generated per launch; the kernel is latency-bound on the sequential MT19937 twist"}


# --------------------------------------------------------------------------- CPU arms
def _oracle_group(args):
    records, seed, policy_dict, resamples = args
    sys.path.insert(0, str(ROOT))
    from oracle import analysis_oracle as O
    res = O.group_summary(records, seed, policy_dict, resamples)
    return sum(1 for _, ci in res if ci) * resamples


def cpu_baseline(records, policy, groups: int = 8) -> dict:
    """The oracle (a restatement of the reference's Python) on one core over a bounded sample."""
    from dataclasses import asdict
    from powermodeling_b200.analysis import group_key
    pol = {k: v for k, v in asdict(policy).items() if k not in ("near_optimum_fraction", "min_geometries")}
    chunks = [records[i * REPEATS:(i + 1) * REPEATS] for i in range(groups)]
    t0 = time.perf_counter()
    total = sum(_oracle_group((c, 1000003 + i, pol, RESAMPLES)) for i, c in enumerate(chunks))
    dt = time.perf_counter() - t0
    return {"value": total / dt, "unit": "resamples/s", "cores": 1, "kind": "port",
            "sample": f"{groups} of {POINTS} points ({groups * REPEATS} trials), B={RESAMPLES}, {dt:.1f} s"}


def run_reference(args) -> dict:
    """The reference's CPU analysis restated (oracle), all host cores, on the same workload."""
    from dataclasses import asdict
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(points=POINTS, repeats=REPEATS), seed=0)
    pol = dict(__import__("oracle.analysis_oracle", fromlist=["DEFAULT_POLICY"]).DEFAULT_POLICY, **ANALYSIS_POLICY)
    cores = os.cpu_count() or 1
    jobs = [(records[i * REPEATS:(i + 1) * REPEATS], 1000003 + i, pol, RESAMPLES) for i in range(POINTS)]
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(args.warmup):
            pool.map(_oracle_group, jobs[:cores])
        times, total = [], 0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            total = sum(pool.map(_oracle_group, jobs))
            times.append(time.perf_counter() - t0)
    step_s = sum(times) / len(times)
    value = total / step_s
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "resamples/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "points": POINTS, "repeats": REPEATS, "resamples": RESAMPLES},
            "cpu_baseline": {"value": value, "unit": "resamples/s", "cores": cores, "kind": "port",
                             "sample": f"full workload per step ({POINTS} groups), processes over groups"},
            "e2e": {"value": value, "unit": "resamples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-arms", action="store_true", help="skip the HBM/tensor/GEMM/SFU arm measurements")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        line = run_b200(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
