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
import datetime
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
WORKLOAD = "analysis: 64 points per GPU x 4 paired repeats, 3 s arms / 1 s idles at 10 ms, B=10000"


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock, power and throttle-reason samples around a measurement.

    Sampling starts (and its first row is awaited) before the measurement;
    with mark_begin()/mark_end() around a timed region, the statistics use
    the rows stamped inside it (the rows nearest to it when it is shorter
    than one interval)."""
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,clocks.mem")

    def __init__(self, index: int, interval_ms: int = 20):
        self.index, self.interval_ms, self.proc, self.path = index, interval_ms, None, None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"pmb200_clocks_{os.getpid()}_{id(self)}.csv"
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        deadline = time.time() + 3.0
        while time.time() < deadline and self.proc.poll() is None:
            if self.path.exists() and self.path.read_text().strip():
                break
            time.sleep(0.01)

    def mark_begin(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = [line.split(", ") for line in self.path.read_text().splitlines() if line.strip()]
        rows = [r for r in rows if len(r) >= 11]
        stamped = []
        for r in rows:
            try:
                stamped.append((datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp(), r))
            except ValueError:
                pass
        window = rows
        if self.t0 is not None and self.t1 is not None and stamped:
            inside = [r for t, r in stamped if self.t0 <= t <= self.t1]
            if inside:
                window = inside
            else:   # region shorter than one interval: the rows on either side of it
                before = [r for t, r in stamped if t < self.t0][-1:]
                after = [r for t, r in stamped if t > self.t1][:1]
                window = before + after or rows
        num = lambda v: v.strip().replace(".", "", 1).isdigit()
        sm = [float(r[2]) for r in window if num(r[2])]
        mx = [float(r[3]) for r in rows if num(r[3])]
        mem = [float(r[10]) for r in window if num(r[10])]
        power = [float(r[4]) for r in window if num(r[4])]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({name for r in window for name, v in zip(names, r[6:10]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "mem_mhz": statistics.median(mem) if mem else None,
                "power_w_median": statistics.median(power) if power else None,
                "reasons": reasons, "samples": len(window), "samples_total": len(rows),
                "interval_ms": self.interval_ms}


# --------------------------------------------------------------------------- workload
def build_workload(rank: int):
    """Records, packed arrays and analyzed trials of one rank's 64-point shard of the sweep."""
    from powermodeling_b200 import analysis as A
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(points=POINTS, repeats=REPEATS), seed=rank, first_point=rank * POINTS)
    policy = A.AnalysisPolicy(**ANALYSIS_POLICY)
    packed, _, _ = A.prepare(records)
    trials = A.analyze_trials(records, policy)              # one untimed pass for the group keys
    return records, policy, packed, trials


def global_groups(trials: list, world: int):
    """Group structure of the whole sweep (every rank's trials, rank order): members as global rows, seeds."""
    from powermodeling_b200 import analysis as A
    if world > 1:
        import torch.distributed as dist
        light = [{k: t.get(k) for k in ("trial_id", "valid", "repeat_index", "config", "gpu_uuid", "workload",
                                        "experiment_role", "clock_comparison_controlled", "graphics_clock_mhz",
                                        "memory_clock_mhz", "benchmark_sha256", "measurement_stratum",
                                        "experiment_contract", "nonlinear_contract", "sfu_contract",
                                        "treatment_design_stratum", "resource_geometry")} for t in trials]
        parts: list = [None] * world
        dist.all_gather_object(parts, light)
        everything = [t for part in parts for t in part]
    else:
        everything = trials
    buckets: dict[str, list[int]] = {}
    for i, t in enumerate(everything):
        buckets.setdefault(A.group_key(t), []).append(i)
    keys = sorted(buckets)
    return [buckets[k] for k in keys], [A.group_seed(k) for k in keys]


def device_arrays(packed, torch):
    from powermodeling_b200 import _native as N
    dev = {}
    t = N.Trials()
    t.n_trials, t.max_phase_samples, t.n_samples, t.n_epochs = packed.n_trials, packed.max_phase_samples, packed.n_samples, packed.n_epochs
    t.broadcast_columns = packed.broadcast
    for name, dtype, _ in N.TRIAL_ARRAYS + N.EPOCH_ARRAYS + N.TAIL_ARRAYS:
        a = packed.arrays[name]
        d = torch.from_numpy(a.copy()).cuda() if a.size else torch.empty(1, dtype=torch.uint8, device="cuda")
        dev[name] = d
        setattr(t, name, d.data_ptr())
    in_bytes = sum(packed.arrays[n].nbytes for n, _, _ in N.TRIAL_ARRAYS + N.EPOCH_ARRAYS + N.TAIL_ARRAYS)
    return t, dev, in_bytes


def run_b200(args, rank: int, world: int) -> dict | None:
    """One step = analyze this rank's trials, exchange metric rows, bootstrap this rank's groups, exchange results."""
    import torch
    import torch.distributed as dist
    from powermodeling_b200 import _native as N
    from powermodeling_b200.analysis import METRICS
    from powermodeling_b200.distributed import owned_groups

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    lib = N.library()
    records, policy, packed, host_trials_list = build_workload(rank)
    members, seeds = global_groups(host_trials_list, world)
    n, M, G = packed.n_trials, len(METRICS), len(members)
    mine = owned_groups(G, world, rank)
    per_rank = -(-G // world)
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
    # Exchange one lands every rank's metric rows and valid flags in the gathered buffers (rank order =
    # global row order): by default the analysis kernel stores them into every rank's buffers over
    # NVLink (peer memory, pmb200_peer.h); with --exchange nccl, an all-gather after it.
    # If the peer exchange cannot be set up, or fails the check against NCCL after the warm-up
    # steps, every rank takes the NCCL form instead and the line says why.
    peer = world > 1 and args.exchange == "peer"
    px, exchange_note = None, None
    if peer:
        from powermodeling_b200.peer import PeerExchange, PeerExchangeError
        try:
            px = PeerExchange(rank, world, n, M, per_rank)
        except PeerExchangeError as exc:
            peer, exchange_note = False, f"NVLink peer exchange not set up ({exc}); NCCL all-gathers used"
    own = [members[g] for g in mine]
    offsets = np.zeros(len(own) + 1, dtype=np.int32)
    np.cumsum([len(m) for m in own], out=offsets[1:])
    rows = np.concatenate([np.asarray(m, dtype=np.int32) for m in own]) if own else np.zeros(1, np.int32)
    d_off, d_rows = torch.from_numpy(offsets).cuda(), torch.from_numpy(rows).cuda()
    own_seeds = np.asarray([seeds[g] for g in mine] or [0], dtype=np.uint64)
    d_seeds = torch.from_numpy(own_seeds.view(np.int64)).cuda()
    # Group outputs of this rank: [3, per_rank, M] (medians, lows, highs); exchange two gathers them.
    group_out = torch.full((3, per_rank, M), float("nan"), dtype=torch.float64, device="cuda")
    max_members = max((len(m) for m in own), default=1)

    def exchange_buffers():
        """Gathered rows, valid flags and group results for the current exchange form, and the job reading them."""
        if peer:
            a_m, a_v, a_g, m_ptr, v_ptr = None, None, None, px.metrics_ptr, px.valid_ptr
        else:
            a_m = torch.empty(world * n * M, dtype=torch.float64, device="cuda") if world > 1 else out["metrics"]
            a_v = torch.empty(world * n, dtype=torch.uint8, device="cuda") if world > 1 else out["valid"]
            a_g = torch.empty((world, 3, per_rank, M), dtype=torch.float64, device="cuda") if world > 1 else None
            m_ptr, v_ptr = a_m.data_ptr(), a_v.data_ptr()
        j = N.BootstrapJob(len(own), M, int(sum(len(m) for m in own)), world * n, RESAMPLES, max_members,
                           m_ptr, d_off.data_ptr(), d_rows.data_ptr(), v_ptr,
                           d_seeds.data_ptr(), group_out[0].data_ptr(), group_out[1].data_ptr(), group_out[2].data_ptr())
        return a_m, a_v, a_g, j

    all_metrics, all_valid, all_group_out, job = exchange_buffers()
    a_scr = lib.pm_analyze_scratch_bytes(n, packed.max_phase_samples)
    b_scr = lib.pm_bootstrap_scratch_bytes(max(1, len(own)), max_members, RESAMPLES)
    scratch = torch.empty(max(1, a_scr + b_scr), dtype=torch.uint8, device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    sptr, side_ptr = C.c_void_p(stream.cuda_stream), C.c_void_p(side.cuda_stream)
    boot_scratch = C.c_void_p(scratch.data_ptr() + a_scr)
    native_policy = policy.native()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    side_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]

    def step():
        # The resample draws need only seeds and group sizes: drawn on a side
        # stream while this rank's trials are analysed and the rows exchanged.
        ev[0].record(stream)
        side.wait_event(ev[0])
        side_ev[0].record(side)
        if own:
            N.check(lib.pm_bootstrap_prepare_device(job, boot_scratch, b_scr, side_ptr), "prepare")
        side_ev[1].record(side)
        if peer:
            px.next_epoch()
            N.check(lib.pm_analyze_trials_device_exchange(trials, native_policy, results, C.c_void_p(scratch.data_ptr()),
                                                          a_scr, C.byref(px.rows), sptr), "analyze + row exchange")
        else:
            N.check(lib.pm_analyze_trials_device(trials, native_policy, results, C.c_void_p(scratch.data_ptr()), a_scr, sptr), "analyze")
        ev[1].record(stream)
        if peer:
            px.wait_rows(stream.cuda_stream)
        elif world > 1:
            dist.all_gather_into_tensor(all_metrics, out["metrics"])
            dist.all_gather_into_tensor(all_valid, out["valid"])
        ev[2].record(stream)
        stream.wait_event(side_ev[1])
        if peer:
            N.check(lib.pm_bootstrap_finish_device_exchange(job, boot_scratch, b_scr, C.byref(px.groups), sptr),
                    "finish + group exchange")
        elif own:
            N.check(lib.pm_bootstrap_finish_device(job, boot_scratch, b_scr, sptr), "finish")
        ev[3].record(stream)
        if peer:
            px.wait_groups(stream.cuda_stream)
        elif world > 1:
            dist.all_gather_into_tensor(all_group_out, group_out)
        ev[4].record(stream)

    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()                                  # every rank launches its first step together
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if peer:
        # The rows and group results the kernels stored into this rank must equal NCCL
        # all-gathers of every rank's own outputs, bit for bit, and no arrival wait may have expired.
        want_rows = torch.empty(world * n * M, dtype=torch.float64, device="cuda")
        want_valid = torch.empty(world * n, dtype=torch.uint8, device="cuda")
        want_groups = torch.empty((world, 3, per_rank, M), dtype=torch.float64, device="cuda")
        dist.all_gather_into_tensor(want_rows, out["metrics"])
        dist.all_gather_into_tensor(want_valid, out["valid"])
        dist.all_gather_into_tensor(want_groups, group_out)
        torch.cuda.synchronize()
        good = (int(px.error.item()) == 0
                and torch.equal(px.view("metrics").reshape(-1).view(torch.int64), want_rows.view(torch.int64))
                and torch.equal(px.view("valid"), want_valid)
                and torch.equal(px.view("groups").reshape(-1).view(torch.int64), want_groups.reshape(-1).view(torch.int64)))
        verdict = torch.tensor([0 if good else 1], dtype=torch.int32, device="cuda")
        dist.all_reduce(verdict, op=dist.ReduceOp.MAX)
        del want_rows, want_valid, want_groups
        if int(verdict.item()):
            px.close()
            px, peer = None, False
            exchange_note = "NVLink peer exchange failed its check against NCCL after the warm-up; NCCL all-gathers used"
            all_metrics, all_valid, all_group_out, job = exchange_buffers()
            for _ in range(args.warmup):
                flush.zero_()
                step()
            torch.cuda.synchronize()
    if peer:
        gathered = px.view("groups").cpu().numpy()
    else:
        gathered = (all_group_out if world > 1 else group_out.unsqueeze(0)).cpu().numpy()
    resamples_per_step = int(np.isfinite(gathered[:, 1]).sum()) * RESAMPLES
    # group g was bootstrapped by rank g % world as its (g // world)-th group
    lo_global = np.stack([gathered[g % world, 1, g // world] for g in range(G)])
    # correctness guard on the timed configuration: every trial valid, every group filled
    assert int(out["valid"].sum().item()) == n, "synthetic trials must all be valid"
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    clocks.mark_begin()
    parts_ms = {"analyze": [], "exchange_rows": [], "join_and_finish": [], "exchange_groups": []}
    prepare_ms, step_ms = [], []
    for _ in range(args.steps):
        flush.zero_()                                   # L2 flush, outside the timed events
        step()
        ev[4].synchronize()
        for k, name in enumerate(parts_ms):
            parts_ms[name].append(ev[k].elapsed_time(ev[k + 1]))
        prepare_ms.append(side_ev[0].elapsed_time(side_ev[1]))
        step_ms.append(ev[0].elapsed_time(ev[4]))
    torch.cuda.synchronize()
    clocks.mark_end()
    clock_info = clocks.stop()
    if world > 1:
        dist.barrier()
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = resamples_per_step / (ms_per_step / 1e3)
    t_analyze, t_boot = parts_ms["analyze"], parts_ms["join_and_finish"]

    # ---- end to end: host buffers through pm_analyze_sweep, then one gather of group results --------
    # Each rank's groups are its own points, so a rank summarizes its shard with one library call
    # (H2D of the packed trials, both kernels, D2H of every result) and the group results are
    # all-gathered (H2D, NCCL, D2H) inside the timed region.
    from powermodeling_b200.pack import trials_struct
    host_trials = trials_struct(packed)
    base = rank * n
    local_groups = [g for g, m in enumerate(members) if m and all(base <= i < base + n for i in m)]
    l_members = [[i - base for i in members[g]] for g in local_groups]
    Gl = len(local_groups)
    l_off = np.zeros(Gl + 1, dtype=np.int32)
    np.cumsum([len(m) for m in l_members], out=l_off[1:])
    l_rows = np.concatenate([np.asarray(m, dtype=np.int32) for m in l_members])
    l_seeds = np.asarray([seeds[g] for g in local_groups], dtype=np.uint64)
    h_out = {"phase_out": np.empty(n * 5 * PO), "phase_flags": np.empty(n * 5, dtype=np.uint32),
             "trial_out": np.empty(n * TO), "issue_bits": np.empty(n * 4, dtype=np.uint64),
             "metrics": np.empty(n * M), "valid": np.empty(n, dtype=np.uint8)}
    h_results = N.TrialResults(*(h_out[k].ctypes.data for k in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid")))
    h_groups = np.empty((3, Gl, M))
    h_job = N.BootstrapJob(Gl, M, int(l_rows.size), n, RESAMPLES, 0, None, l_off.ctypes.data, l_rows.ctypes.data, None,
                           l_seeds.ctypes.data, h_groups[0].ctypes.data, h_groups[1].ctypes.data, h_groups[2].ctypes.data)
    g_send = torch.empty((3, Gl, M), dtype=torch.float64, device="cuda")
    g_recv = torch.empty((world, 3, Gl, M), dtype=torch.float64, device="cuda")

    def e2e_step():
        N.check(lib.pm_analyze_sweep(host_trials, native_policy, h_results, h_job), "pm_analyze_sweep")
        if world > 1:
            g_send.copy_(torch.from_numpy(h_groups))
            dist.all_gather_into_tensor(g_recv, g_send)
            return g_recv.cpu().numpy()
        return h_groups[None]

    for _ in range(args.warmup):
        e2e_step()
    if world > 1:
        dist.barrier()
    e2e_times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        e2e_step()
        e2e_times.append(time.perf_counter() - t0)
    e2e_s = sum(e2e_times) / args.steps
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    assert np.array_equal(np.nan_to_num(h_groups[1]), np.nan_to_num(lo_global[local_groups])), \
        "e2e and device paths disagree"
    if peer:
        px.check()
        px.close()
    h2d = in_bytes + l_off.nbytes + l_rows.nbytes + l_seeds.nbytes + (h_groups.nbytes if world > 1 else 0)
    d2h = sum(a.nbytes for a in h_out.values()) + h_groups.nbytes * (world + 1 if world > 1 else 1)
    if rank != 0:
        return None
    peaks = measured_peaks()
    a_ms, b_ms = statistics.mean(t_analyze), statistics.mean(t_boot)
    dominant = "bootstrap_kernel" if b_ms >= a_ms else "analyze_kernel"
    roofline = roofline_entry(dominant, a_ms, b_ms, in_bytes, out_bytes, len(own), M, packed, peaks,
                              resamples_per_step)
    line = {"metric": METRIC, "value": value, "unit": "resamples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "points": POINTS * world, "points_per_gpu": POINTS, "repeats": REPEATS,
                       "trials": n * world, "groups": G,
                       "resamples": RESAMPLES, "samples": packed.n_samples, "l2": "flushed (256 MiB write) between steps",
                       "parallelism": (f"sweep-sharded x{world}: trials and groups per rank; metric rows and group "
                                       f"results stored into every rank by the analysis and bootstrap kernels over "
                                       f"NVLink peer memory" if peer else
                                       f"sweep-sharded x{world}: trials and groups per rank, rows and group results "
                                       f"all-gathered over NCCL") if world > 1 else "single GPU"},
            "e2e": {"value": resamples_per_step / e2e_s, "unit": "resamples/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_s * 1e3},
            # per step: analyze, the draws and the finish (or, owning no group, analyze and the
            # group signal), plus the two arrival waits of the peer exchange
            "gpu_launches": ((3 if own else 2) if peer else (3 if own else 1)) * args.steps + (2 * args.steps if peer else 0),
            "kernels": {"analyze_kernel_ms": a_ms,
                        "bootstrap_prepare_kernel_ms (side stream, overlaps analyze)": statistics.mean(prepare_ms),
                        "join_and_bootstrap_finish_ms": b_ms,
                        ("rows_arrival_wait_ms" if peer else "exchange_rows_ms"): statistics.mean(parts_ms["exchange_rows"]),
                        "exchange_groups_ms": statistics.mean(parts_ms["exchange_groups"])},
            "roofline": roofline, "clocks": clock_info}
    if world > 1:
        line["exchange"] = "nvlink-peer" if peer else "nccl"
        if exchange_note:
            line["exchange_note"] = exchange_note
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(records, policy)
    if not args.no_arms and world == 1:
        line["arms"] = run_arms(local, peaks)
        line["arms"]["analysis_scaled"] = run_scaled_analysis(packed, native_policy, peaks)
    return line


def replicate_packed(packed, copies: int):
    """The packed batch repeated `copies` times (offsets rebased; broadcast columns stay one element)."""
    from types import SimpleNamespace
    from powermodeling_b200 import _native as N
    a, k = packed.arrays, copies
    out = {}
    for name, _, key in N.TRIAL_ARRAYS + N.EPOCH_ARRAYS + N.TAIL_ARRAYS:
        x = a[name]
        if name in ("phase_offsets", "epoch_offsets"):
            step = packed.n_samples if name == "phase_offsets" else packed.n_epochs
            out[name] = np.concatenate([x[:-1] + c * step for c in range(k)] + [x[-1:] + (k - 1) * step]).astype(x.dtype)
        elif key == "samples" and x.size == 1 and packed.n_samples > 1:
            out[name] = x
        else:
            out[name] = np.tile(x, k)
    return SimpleNamespace(arrays=out, n_trials=packed.n_trials * k, n_samples=packed.n_samples * k,
                           n_epochs=packed.n_epochs * k, max_phase_samples=packed.max_phase_samples,
                           broadcast=packed.broadcast)


def run_scaled_analysis(packed, native_policy, peaks: dict) -> dict:
    """The analysis kernel alone on the sweep repeated up to 65 536 trials (16 384 points): trials
    integrated per second and input bytes read per second as the batch outgrows the L2."""
    import torch
    from powermodeling_b200 import _native as N
    lib = N.library()
    PO, TO, M = N.layout("PM_PO_COUNT"), N.layout("PM_TO_COUNT"), N.layout("PM_M_COUNT")
    stream = torch.cuda.current_stream()
    sptr = C.c_void_p(stream.cuda_stream)
    hbm = peaks.get("hbm_gbs", 6650.0)
    out = {}
    for copies in (1, 16, 64, 256):
        big = replicate_packed(packed, copies)
        trials, keep, in_bytes = device_arrays(big, torch)
        n = big.n_trials
        res = {"phase_out": torch.empty(n * 5 * PO, dtype=torch.float64, device="cuda"),
               "phase_flags": torch.empty(n * 5, dtype=torch.int32, device="cuda"),
               "trial_out": torch.empty(n * TO, dtype=torch.float64, device="cuda"),
               "issue_bits": torch.empty(n * 4, dtype=torch.int64, device="cuda"),
               "metrics": torch.empty(n * M, dtype=torch.float64, device="cuda"),
               "valid": torch.empty(n, dtype=torch.uint8, device="cuda")}
        results = N.TrialResults(*(res[k].data_ptr() for k in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid")))
        out_bytes = sum(v.numel() * v.element_size() for v in res.values())
        scr_n = lib.pm_analyze_scratch_bytes(n, big.max_phase_samples)
        scr = torch.empty(max(1, scr_n), dtype=torch.uint8, device="cuda")
        run = lambda: N.check(lib.pm_analyze_trials_device(trials, native_policy, results, C.c_void_p(scr.data_ptr()),
                                                             scr_n, sptr), "analyze (scaled)")
        for _ in range(3):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            run()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        assert int(res["valid"].sum().item()) == n, "replicated trials must all be valid"
        gbs = (in_bytes + out_bytes) / (ms / 1e3) / 1e9
        out[str(n)] = {"points": n // 4, "ms": ms, "trials_per_s": n / (ms / 1e3), "samples_per_s": big.n_samples / (ms / 1e3),
                       "algorithmic_gbs": gbs, "frac_of_hbm": gbs / hbm, "input_bytes": int(in_bytes)}
        del trials, keep, res, scr
    return out


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
    out["nonlinear"] = run_nonlinear_arms(sms, peaks)
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


NONLINEAR_ELEMENTS = 1 << 28          # 1 GiB of fp32 input, 1 GiB of output: far above the 126 MB L2
NONLINEAR_ROW_WIDTH = 1024            # the reference's default row width


def run_nonlinear_arms(sms: int, peaks: dict) -> dict:
    """The complete FP32 nonlinear functions through powerbench at HBM scale.

    Each arm: 2^28 inputs, fixed grid of 8 CTAs x 256 threads per SM, one
    application per launch, 8 launches per batch.  ``logical_gbs`` is the
    reference's count (8 B per element pointwise, 16 B row-wise: x read two
    or three times); ``hbm_gbs`` counts what the algorithm must move, x once
    and y once (8 B per element; RMSNorm's gamma row stays in L2), against the
    measured copy peak."""
    hbm = peaks.get("hbm_gbs", 6650.0)
    out = {}
    for fn in ("exp", "tanh", "silu", "rmsnorm", "softmax"):
        args = ["--workload", fn, "--nonlinear-mode", "streaming", "--grid-mode", "fixed", "--blocks", str(sms * 8),
                "--threads", "256", "--working-set-bytes", str(NONLINEAR_ELEMENTS * 4), "--iterations", "1",
                "--batch-launches", "8", "--fixed-batches", "6", *ARM_QUICK]
        if fn in ("rmsnorm", "softmax"):
            args += ["--row-width", str(NONLINEAR_ROW_WIDTH)]
        _, r = _arm(args)
        algorithmic = r["elements"] * 8 / r["duration_s"] / 1e9
        out[fn] = {"elements_s": r["throughput_ops_s"], "logical_gbs": r["throughput_bytes_s"] / 1e9,
                   "hbm_gbs": algorithmic, "frac_of_measured_copy_peak": algorithmic / hbm,
                   "validation_passed": r["sanity"]["numerical_validation_passed"], "checksum": r["checksum"],
                   "ms_per_launch": r["duration_s"] / r["kernel_launches"] * 1e3,
                   "config": f"2^28 fp32 inputs, grid {sms}x8x256" + (f", rows of {NONLINEAR_ROW_WIDTH}" if fn in ("rmsnorm", "softmax") else "")}
    return out


# DRAM bytes (read + write) per launch from one ncu capture of the same
# workload (profiles/analysis_sweep_64x4_B10000.md); None where none was taken.
NCU_TRAFFIC_BYTES = {"analyze_kernel": 5_149_184, "bootstrap_kernel": 183_040}


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
    # Each step is a bounded sample of the sweep: one group per host core, the
    # groups taken in turn, so K steps end within minutes on any core count.
    per_step = max(1, min(POINTS, cores))
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(args.warmup):
            pool.map(_oracle_group, jobs[:per_step])
        times, resamples = [], 0
        for k in range(args.steps):
            batch = [jobs[(k * per_step + j) % POINTS] for j in range(per_step)]
            t0 = time.perf_counter()
            resamples += sum(pool.map(_oracle_group, batch))
            times.append(time.perf_counter() - t0)
    step_s = sum(times) / len(times)
    value = resamples / sum(times)
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "resamples/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "points": POINTS * max(1, args.gpus), "points_per_gpu": POINTS,
                       "repeats": REPEATS, "resamples": RESAMPLES},
            "cpu_baseline": {"value": value, "unit": "resamples/s", "cores": cores, "kind": "port",
                             "sample": f"{per_step} of the {POINTS} groups per step (one per core, in turn), "
                                       f"processes over groups"},
            "e2e": {"value": value, "unit": "resamples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--exchange", choices=("peer", "nccl"), default="peer",
                        help="N>1: metric rows stored into every rank by the analysis kernel over NVLink, or all-gathered by NCCL")
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
