"""Benchmark of the analysis hot path: bootstrap resamples per second.

Workload: 64 sweep points x 4 repeats of paired trials (3 s arms, 1 s idles,
10 ms samples with 0-2 ms jitter, N(450,15)/N(300,10)/N(90,3) W), seed 0 per
rank; one step analyzes every trial (phase integrals over aligned epochs,
idle-delta, paired pJ/FLOP) and computes every group's medians and
10 000-draw percentile-bootstrap intervals.  ``value`` counts
resamples = sum over groups of (metrics with an interval) x B per second of
device time with inputs resident in HBM (L2 flushed between steps); ``e2e``
is the same metric through the drop-in call summarize(records) on the
runner's record dicts, and ``e2e_c_abi`` through the host-buffer C-ABI call
pm_analyze_sweep on packed arrays.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
Under torchrun each rank analyzes its own 64 points and bootstraps their
groups (weak scaling); the group results are gathered on rank 0 every step;
device time is the maximum over ranks.
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


class GpuClockWatch:
    """This rank's GPU: SM clock and clock-event reasons read every 0.1 ms by a native thread
    (telemetry.ClockWatch) while the timed steps run, so a region of a few milliseconds has
    many clock records (nvidia-smi's loop gives one every 20 ms)."""
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, local: int):
        self.device = self.watch = None
        try:
            from powermodeling_b200 import powerbench
            from powermodeling_b200.telemetry import ClockWatch, NvmlDevice
            uuid = next(r for r in powerbench.run(["--describe", "--device", str(local)]) if r["type"] == "device")["uuid"]
            self.device = NvmlDevice(uuid=uuid)
            self.watch = ClockWatch(self.device, interval_s=1e-4)
        except Exception:                               # no NVML here: the nvidia-smi record stands alone
            self.device = self.watch = None

    def start(self):
        """Started ahead of the timed steps: the thread's first reads of a newly opened device
        take milliseconds, longer than a short timed region."""
        if self.watch:
            self.watch.start()

    def stop(self, begin: float, end: float) -> dict | None:
        """The records read between ``begin`` and ``end`` (time.monotonic(), the watch's clock);
        the one nearest the region when none falls inside it."""
        if not self.watch:
            return None
        try:
            t, mhz, bits = self.watch.stop()
        finally:
            self.device.close()
        if not len(t):
            return None
        inside = (t >= begin) & (t <= end)
        if inside.any():
            t, mhz, bits = t[inside], mhz[inside], bits[inside]
        else:
            nearest = int(np.argmin(np.minimum(np.abs(t - begin), np.abs(t - end))))
            t, mhz, bits = t[nearest:nearest + 1], mhz[nearest:nearest + 1], bits[nearest:nearest + 1]
        union = 0
        for b in set(bits.tolist()):
            union |= int(b)
        return {"sm_mhz": float(statistics.median(mhz.tolist())), "sm_mhz_min": int(mhz.min()), "samples": int(len(t)),
                "reasons": sorted(name for bit, name in self.REASONS.items() if union & bit)}


def merge_clock_records(records: list) -> dict | None:
    """One clock record for all ranks: the median of the ranks' medians, the lowest clock seen,
    every reason seen, and the samples counted over all GPUs."""
    records = [r for r in records if r]
    if not records:
        return None
    return {"sm_mhz": statistics.median(r["sm_mhz"] for r in records), "sm_mhz_min": min(r["sm_mhz_min"] for r in records),
            "samples": sum(r["samples"] for r in records), "gpus": len(records),
            "reasons": sorted({x for r in records for x in r["reasons"]}),
            "source": "native NVML clock watch, every 0.1 ms on each GPU during the timed steps"}


# --------------------------------------------------------------------------- workload
def build_workload(rank: int, world: int = 1, strong: bool = False):
    """Records, packed arrays and analyzed trials of one rank's share of the sweep: its own 64 points
    (weak scaling), or its slice of one 64-point sweep, whole points only (strong scaling)."""
    from powermodeling_b200 import analysis as A
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    if strong:
        lo, hi = rank * POINTS // world, (rank + 1) * POINTS // world
        records = [r for r in make_sweep(SweepShape(points=POINTS, repeats=REPEATS), seed=0)
                   if lo <= r["config"]["point"] < hi]
    else:
        records = make_sweep(SweepShape(points=POINTS, repeats=REPEATS), seed=rank, first_point=rank * POINTS)
    policy = A.AnalysisPolicy(**ANALYSIS_POLICY)
    packed, _, _ = A.prepare(records)
    trials = A.analyze_trials(records, policy)              # one untimed pass for the group keys
    return records, policy, packed, trials


def local_groups(trials: list):
    """Groups of this rank's own trials (key order): member rows, sha256 seeds.

    Every group is bootstrapped on the rank that analysed its members (the
    sweep's points are partitioned over ranks), so no metric row leaves its GPU."""
    from powermodeling_b200 import analysis as A
    buckets: dict[str, list[int]] = {}
    for i, t in enumerate(trials):
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
    """One step = analyze this rank's trials, bootstrap this rank's groups, gather the group results on rank 0."""
    import torch
    import torch.distributed as dist
    from powermodeling_b200 import _native as N
    from powermodeling_b200.analysis import METRICS

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    lib = N.library()
    strong = args.scaling == "strong"
    records, policy, packed, host_trials_list = build_workload(rank, world, strong)
    members, seeds = local_groups(host_trials_list)
    n, M, G = packed.n_trials, len(METRICS), len(members)
    per_rank = G
    if world > 1:
        most = torch.tensor([G], dtype=torch.int64, device="cuda")
        dist.all_reduce(most, op=dist.ReduceOp.MAX)
        per_rank = int(most.item())
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
    # Groups are owned by the rank that analysed their members, so the only
    # exchange is the gather of every rank's group results on rank 0: by
    # default the finish kernel stores them into rank 0's gathered buffer over
    # NVLink (peer memory, pmb200_peer.h) and rank 0's stream waits for every
    # rank's arrival flag of the step; with --exchange nccl, an all-gather.
    # If the peer gather cannot be set up, or fails the check against NCCL
    # after the warm-up steps, every rank takes the NCCL form instead and the
    # line says why.
    peer = world > 1 and args.exchange == "peer"
    px, exchange_note = None, None
    if peer:
        from powermodeling_b200.peer import PeerExchange, PeerExchangeError
        try:
            px = PeerExchange(rank, world, 0, M, per_rank, root=0)
        except PeerExchangeError as exc:
            peer, exchange_note = False, f"NVLink peer gather not set up ({exc}); NCCL all-gathers used"
    offsets = np.zeros(G + 1, dtype=np.int32)
    np.cumsum([len(m) for m in members], out=offsets[1:])
    rows = np.concatenate([np.asarray(m, dtype=np.int32) for m in members]) if members else np.zeros(1, np.int32)
    d_off, d_rows = torch.from_numpy(offsets).cuda(), torch.from_numpy(rows).cuda()
    d_seeds = torch.from_numpy(np.asarray(seeds or [0], dtype=np.uint64).view(np.int64)).cuda()
    # Group outputs of this rank: [3, per_rank, M] (medians, lows, highs).
    group_out = torch.full((3, per_rank, M), float("nan"), dtype=torch.float64, device="cuda")
    all_group_out = torch.full((world, 3, per_rank, M), float("nan"), dtype=torch.float64, device="cuda") if world > 1 else None
    max_members = max((len(m) for m in members), default=1)
    job = N.BootstrapJob(G, M, int(sum(len(m) for m in members)), n, RESAMPLES, max_members,
                         out["metrics"].data_ptr(), d_off.data_ptr(), d_rows.data_ptr(), out["valid"].data_ptr(),
                         d_seeds.data_ptr(), group_out[0].data_ptr(), group_out[1].data_ptr(), group_out[2].data_ptr())
    a_scr = lib.pm_analyze_scratch_bytes(n, packed.max_phase_samples)
    b_scr = lib.pm_bootstrap_scratch_bytes(max(1, G), max_members, RESAMPLES)
    sweep_scr = lib.pm_analyze_sweep_scratch_bytes(n, packed.max_phase_samples, G, max_members, RESAMPLES)
    scratch = torch.empty(max(1, a_scr + b_scr, sweep_scr), dtype=torch.uint8, device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    sptr, side_ptr = C.c_void_p(stream.cuda_stream), C.c_void_p(side.cuda_stream)
    boot_scratch = C.c_void_p(scratch.data_ptr() + a_scr)
    native_policy = policy.native()
    scratch_ptr, scratch_bytes = C.c_void_p(scratch.data_ptr()), scratch.numel()

    def step(ev):
        # One call per step: the library forks the draws onto its side stream
        # beside the analysis, joins them and runs the finish (with the group
        # gather's peer stores when it is on); rank 0 then waits for every
        # rank's arrival flag of the step, or the ranks all-gather over NCCL.
        ev[0].record(stream)
        if peer:
            px.next_epoch()
        N.check(lib.pm_analyze_sweep_device(trials, native_policy, results, job, scratch_ptr, scratch_bytes,
                                            C.byref(px.groups) if peer else None, sptr), "pm_analyze_sweep_device")
        if peer:
            if rank == 0:
                px.wait_groups(stream.cuda_stream)
        elif world > 1:
            dist.all_gather_into_tensor(all_group_out, group_out)
        ev[1].record(stream)

    def run_steps(k):
        """k steps enqueued back to back (L2 flushed before each, outside its events); no host wait between them."""
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(k)]
        if peer:
            px.gate(stream.cuda_stream)                 # every rank's GPU starts the steps together
        for i in range(k):
            flush.zero_()
            step(evs[i])
        return evs

    def breakdown(k):
        """Per-kernel times of k further steps through the separate entry points, each step
        enqueued whole before the GPU reaches it (a synchronize, then the L2 flush, ahead of it):
        the analysis, the draws on the side stream beside it, the join and the finish."""
        parts = {"analyze": [], "prepare": [], "join": [], "finish": []}
        for _ in range(k):
            torch.cuda.synchronize()
            flush.zero_()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            sev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            ev[0].record(stream)
            side.wait_event(ev[0])
            sev[0].record(side)
            if G:
                N.check(lib.pm_bootstrap_prepare_device(job, boot_scratch, b_scr, side_ptr), "prepare")
            sev[1].record(side)
            N.check(lib.pm_analyze_trials_device(trials, native_policy, results, C.c_void_p(scratch.data_ptr()), a_scr,
                                                 sptr), "analyze")
            ev[1].record(stream)
            stream.wait_event(sev[1])
            ev[2].record(stream)
            if G:
                N.check(lib.pm_bootstrap_finish_device(job, boot_scratch, b_scr, sptr), "finish")
            ev[3].record(stream)
            torch.cuda.synchronize()
            parts["analyze"].append(ev[0].elapsed_time(ev[1]))
            parts["prepare"].append(sev[0].elapsed_time(sev[1]))
            parts["join"].append(ev[1].elapsed_time(ev[2]))
            parts["finish"].append(ev[2].elapsed_time(ev[3]))
        return {k: statistics.median(v) for k, v in parts.items()}

    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
    run_steps(args.warmup)
    torch.cuda.synchronize()
    if peer:
        # The group results the kernels stored into rank 0 must equal an NCCL
        # all-gather of every rank's own outputs, bit for bit (each rank's owned
        # slots), and no arrival wait may have expired.
        want_groups = torch.empty((world, 3, per_rank, M), dtype=torch.float64, device="cuda")
        dist.all_gather_into_tensor(want_groups, group_out)
        counts = torch.tensor([G], dtype=torch.int64, device="cuda")
        all_counts = torch.empty(world, dtype=torch.int64, device="cuda")
        dist.all_gather_into_tensor(all_counts, counts)
        torch.cuda.synchronize()
        good = int(px.error.item()) == 0
        if rank == 0:
            got = px.view("groups")
            for r in range(world):
                c = int(all_counts[r].item())
                good = good and torch.equal(got[r, :, :c].reshape(-1).view(torch.int64),
                                            want_groups[r, :, :c].reshape(-1).view(torch.int64))
        verdict = torch.tensor([0 if good else 1], dtype=torch.int32, device="cuda")
        dist.all_reduce(verdict, op=dist.ReduceOp.MAX)
        del want_groups
        if int(verdict.item()):
            px.close()
            px, peer = None, False
            exchange_note = "NVLink peer gather failed its check against NCCL after the warm-up; NCCL all-gathers used"
            run_steps(args.warmup)
            torch.cuda.synchronize()
    # correctness guard on the timed configuration: every trial valid
    assert int(out["valid"].sum().item()) == n, "synthetic trials must all be valid"
    finite = torch.tensor([int(np.isfinite(group_out[1].cpu().numpy()).sum())], dtype=torch.int64, device="cuda")
    if world > 1:
        dist.all_reduce(finite)
    resamples_per_step = int(finite.item()) * RESAMPLES
    lo_local = group_out[1].cpu().numpy()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(",".join(str(i) for i in range(world))) if rank == 0 else None
    if clocks:
        clocks.start()
    watch = GpuClockWatch(local)
    watch.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.mark_begin()
    begin = time.monotonic()
    evs = run_steps(args.steps)
    torch.cuda.synchronize()
    end = time.monotonic()
    if clocks:
        clocks.mark_end()
    watched = watch.stop(begin, end)
    if world > 1:
        everyone: list = [None] * world
        dist.all_gather_object(everyone, watched)
        watched = merge_clock_records(everyone)
    else:
        watched = merge_clock_records([watched])
    clock_info = clocks.stop() if clocks else None
    if rank == 0 and watched:
        clock_info = dict(clock_info or {}, nvidia_smi_samples=(clock_info or {}).get("samples"),
                          sm_mhz=watched["sm_mhz"], sm_mhz_min=watched["sm_mhz_min"],
                          reasons=sorted(set(watched["reasons"]) | set((clock_info or {}).get("reasons") or [])),
                          samples=watched["samples"], source=watched["source"])
    step_ms = [ev[0].elapsed_time(ev[1]) for ev in evs]
    parts = breakdown(50)                               # untimed: the kernels of the step one by one
    if world > 1:
        dist.barrier()
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    n_total, g_total = n * world, G * world
    if world > 1:
        sizes = torch.tensor([n, G], dtype=torch.int64, device="cuda")
        dist.all_reduce(sizes)
        n_total, g_total = int(sizes[0].item()), int(sizes[1].item())
    value = resamples_per_step / (ms_per_step / 1e3)

    # ---- end to end ------------------------------------------------------------------------------
    # e2e: the drop-in call itself, summarize(records) (analysis.py:1400), on the runner's record
    # dicts: record checks and packing, H2D, both kernels, D2H, issue strings and the trial and
    # group dicts.  Each rank summarizes its own points (weak scaling).
    # e2e_c_abi: the same numeric work through the host-buffer C-ABI call pm_analyze_sweep on the
    # packed arrays (H2D of the packed trials and group inputs, D2H of every result).
    from powermodeling_b200 import analysis as A
    from powermodeling_b200.pack import trials_struct
    host_trials = trials_struct(packed)
    h_out = {"phase_out": np.empty(n * 5 * PO), "phase_flags": np.empty(n * 5, dtype=np.uint32),
             "trial_out": np.empty(n * TO), "issue_bits": np.empty(n * 4, dtype=np.uint64),
             "metrics": np.empty(n * M), "valid": np.empty(n, dtype=np.uint8)}
    h_results = N.TrialResults(*(h_out[k].ctypes.data for k in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid")))
    h_groups = np.empty((3, G, M))
    h_seeds = np.asarray(seeds, dtype=np.uint64)
    h_job = N.BootstrapJob(G, M, int(rows.size), n, RESAMPLES, 0, None, offsets.ctypes.data, rows.ctypes.data, None,
                           h_seeds.ctypes.data, h_groups[0].ctypes.data, h_groups[1].ctypes.data, h_groups[2].ctypes.data)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        if world > 1:
            dist.barrier()
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        mean = sum(times) / len(times)
        if world > 1:
            t = torch.tensor([mean], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            mean = float(t.item())
        return mean

    c_abi_s = timed(lambda: N.check(lib.pm_analyze_sweep(host_trials, native_policy, h_results, h_job), "pm_analyze_sweep"))
    assert np.array_equal(np.nan_to_num(h_groups[1]), np.nan_to_num(lo_local[:G])), "C-ABI and device paths disagree"
    summary = {}

    def api_step():
        summary["last"] = A.summarize(records, policy=policy, resamples=RESAMPLES)

    api_s = timed(api_step)
    api_groups = summary["last"]["groups"]
    assert len(api_groups) == G
    for g, group in enumerate(api_groups):
        for m, metric in enumerate(METRICS):
            ci = group["ci95"].get(metric)
            want = lo_local[g, m]
            assert (ci is None and not np.isfinite(want)) or (ci is not None and ci[0] == want), \
                f"summarize and device paths disagree (group {g}, {metric})"
    if peer:
        px.check()
        px.close()
    fleet = run_fleet_arms(local, world, rank) if world > 1 and not args.no_arms else None
    c_h2d = in_bytes + offsets.nbytes + rows.nbytes + h_seeds.nbytes
    c_d2h = sum(a.nbytes for a in h_out.values()) + h_groups.nbytes
    # summarize uploads the packed trials, then the metric and memory-rail rows with the group
    # inputs, and reads back every trial result and every group's medians and interval ends.
    width = M + len(A.SENSOR_FIELDS)
    api_h2d = in_bytes + n * width * 8 + offsets.nbytes + rows.nbytes + h_seeds.nbytes
    api_d2h = sum(a.nbytes for a in h_out.values()) + 3 * G * width * 8
    if rank != 0:
        return None
    peaks = measured_peaks()
    a_ms, f_ms, p_ms = parts["analyze"], parts["finish"], parts["prepare"]
    roofline = roofline_entry(a_ms, p_ms, f_ms, in_bytes, out_bytes, G, M, packed, peaks,
                              (clock_info or {}).get("sm_mhz"))
    line = {"metric": METRIC, "value": value, "unit": "resamples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD if not strong else
                       "analysis: one 64-point sweep split over the GPUs by points, 4 paired repeats, 3 s arms / 1 s idles at 10 ms, B=10000",
                       "points": POINTS if strong else POINTS * world,
                       "points_per_gpu": POINTS // world if strong else POINTS, "repeats": REPEATS,
                       "trials": n_total, "groups": g_total,
                       "resamples": RESAMPLES, "samples": packed.n_samples, "l2": "flushed (256 MiB write) between steps",
                       "parallelism": (f"sweep-partitioned x{world}: each rank analyses its points and bootstraps their "
                                       f"groups; group results gathered on rank 0 " +
                                       ("by the finish kernel's NVLink peer stores" if peer else "by NCCL all-gathers"))
                       if world > 1 else "single GPU"},
            "e2e": {"value": resamples_per_step / api_s, "unit": "resamples/s",
                    "h2d_bytes_per_step": int(api_h2d), "d2h_bytes_per_step": int(api_d2h), "ms_per_step": api_s * 1e3,
                    "call": "summarize(records): record dicts in, summary dicts out"},
            "e2e_c_abi": {"value": resamples_per_step / c_abi_s, "unit": "resamples/s", "h2d_bytes_per_step": int(c_h2d),
                          "d2h_bytes_per_step": int(c_d2h), "ms_per_step": c_abi_s * 1e3,
                          "call": "pm_analyze_sweep on packed host arrays"},
            # per step: the draws, the analysis and the finish, plus rank 0's arrival wait of the peer
            # gather (and the start gate once)
            "gpu_launches": 3 * args.steps + ((args.steps if rank == 0 else 0) + 1 if peer else 0),
            "kernels": {"source": "50 further steps, each enqueued whole before it runs (medians)",
                        "analyze_kernel_ms": a_ms,
                        "bootstrap_prepare_kernel_ms (side stream, overlaps the analysis)": p_ms,
                        "join_wait_ms": parts["join"], "bootstrap_finish_kernel_ms": f_ms},
            "roofline": roofline, "clocks": clock_info}
    if world > 1:
        line["exchange"] = "nvlink-peer" if peer else "nccl"
        if exchange_note:
            line["exchange_note"] = exchange_note
    if fleet:
        line["arms_per_gpu"] = fleet
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(records, policy)
    if not args.no_arms and world == 1:
        arms, detail = run_arms(local, peaks, energy=not args.no_energy)
        scaled = run_scaled_analysis(packed, native_policy, peaks)
        detail["analysis_scaled"] = scaled
        largest = scaled[max(scaled, key=int)]
        arms["analysis_kernel_65536_trials"] = {"trials_per_s": _sig(largest["trials_per_s"]),
                                                "samples_per_s": _sig(largest["samples_per_s"]),
                                                "frac_of_hbm": _sig(largest["frac_of_hbm"], 3)}
        if args.arms_detail:
            Path(args.arms_detail).write_text(json.dumps(detail, indent=1, default=str))
        line["arms"] = arms
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


def _sig(x, digits: int = 4):
    """A float rounded to a few significant digits (the JSON line stays short)."""
    if not isinstance(x, float) or x != x or x in (float("inf"), float("-inf")) or x == 0:
        return x
    from math import floor, log10
    return round(x, max(0, digits - 1 - int(floor(log10(abs(x))))))


def compact(obj, digits: int = 5, keep=("value", "ms_per_step")):
    """The result line with every nested float rounded (the driver keeps the tail of stdout),
    except the headline keys."""
    if isinstance(obj, dict):
        return {k: (v if k in keep else compact(v, digits, ())) for k, v in obj.items()}
    if isinstance(obj, list):
        return [compact(v, digits, ()) for v in obj]
    return _sig(obj, digits) if isinstance(obj, float) else obj


def run_arms(local: int, peaks: dict, energy: bool = True) -> dict:
    """The workload arms on this GPU (powermodeling_b200.sweeps, quick grids): HBM read/copy against the
    interface ceiling, tcgen05 and cuBLAS tensor throughput, the six SFU opcodes at 148 x 8 CTAs,
    L1 and the dependent chase at 96 MiB, and NVML energy per byte, per FLOP and per SFU instruction
    from captured 10 s trials.  Returns (compact summary, full detail)."""
    from powermodeling_b200 import sweeps as S
    dev = S.describe()
    sms, bus = dev["sm_count"], dev["memory_bus_width_bits"]
    clocks = ClockSampler(local)
    clocks.start()
    hbm = S.hbm_sweep(sms, quick=True)
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
    _, r = _arm(["--workload", "gemm", "--gemm-m", "8192", "--gemm-n", "8192", "--gemm-k", "8192", "--batch-launches", "4",
                 "--fixed-batches", "3", *ARM_QUICK])
    gemm_tflops = r["throughput_ops_s"] / 1e12
    sfu = S.sfu_sweep(sms, ks=(8,))
    cache = S.cache_sweep(sms, quick=True)
    nonlinear = run_nonlinear_arms(sms, peaks)
    clock = clocks.stop()
    mem_mhz = clock.get("mem_mhz") or dev["nominal_max_memory_clock_khz"] / 1e3
    sm_mhz = clock.get("sm_mhz") or 1965.0
    S.with_theory(hbm, mem_mhz)
    S.per_sm_clock(sfu, sms, sm_mhz)
    telemetry = run_telemetry_arm(dev["uuid"])
    energy_rows = S.energy_arms(sms) if energy else {}
    dense_peak = 8192 * sms * sm_mhz * 1e6 / 1e12
    best = max(v["tflops"] for v in tensor.values())
    hbm_by = {row["factor"]: row for row in hbm}
    summary = {
        "hbm": {k: {"gbs": _sig(v["gbs"]), "frac_of_theory": _sig(v["frac_of_theory"], 3),
                    "frac_of_measured_copy_peak": _sig(v["gbs"] / peaks.get("hbm_gbs", 6650.0), 3)}
                for k, v in (("read_16B_cs_4GiB", hbm_by["base"]), ("copy_16B_4GiB", hbm_by["access"]),
                             ("read_4B_cg_4GiB", hbm_by["scalar"]), ("read_16B_cs_lcg_fill", hbm_by["fill"]))},
        "hbm_theory_gbs": _sig(2 * mem_mhz * 1e6 * bus / 8 / 1e9),
        "tensor_tcgen05": {"best_tflops": _sig(best), "best_frac_of_dense_peak_at_clock": _sig(max(
            (v.get("frac_of_dense_peak_at_arm_clock") or 0) for v in tensor.values()), 3),
            "frac_of_measured_bf16_gemm": _sig(best / peaks.get("bf16_tflops", 1590.0), 3),
            "by_accumulators_tflops": {k: _sig(v["tflops"]) for k, v in tensor.items()}},
        "gemm_cublas_8192_tflops": _sig(gemm_tflops),
        "sfu_148x8_ops_per_sm_clk": {row["opcode"]: _sig(row["ops_per_sm_per_clock"], 3) for row in sfu},
        "l1_ca_192KiB_per_sm_gbs": _sig(cache["l1"][0]["gbs"]),
        "chase_96MiB_cycles_per_access": {row["granularity"]: _sig(row["cycles_per_access_median"])
                                          for row in cache["chase"]},
        "nonlinear_frac_of_copy_peak": {k: _sig(v["frac_of_measured_copy_peak"], 3) for k, v in nonlinear.items()},
        "telemetry_samples_per_s_at_10ms": _sig(telemetry["interval_10ms"]["samples_per_s"], 3),
    }
    if energy_rows:
        e_hbm, e_tc = energy_rows["hbm_read"], energy_rows["tensor_tcgen05"]
        e_sfu = energy_rows.get("sfu_ex2_paired") or {}
        summary["energy_nvml_10s"] = {
            "hbm_read_pj_per_byte": _sig(e_hbm.get("pj_per_logical_byte")),
            "hbm_read_total_pj_per_byte": _sig(e_hbm.get("total_pj_per_logical_byte")),
            "tcgen05_pj_per_flop": _sig(e_tc.get("operational_idle_increment_pj_per_flop")),
            "tcgen05_total_pj_per_flop": _sig(e_tc.get("total_pj_per_flop")),
            "sfu_ex2_delta_pj_per_instruction": _sig(e_sfu.get("sfu_reference_delta_pj_per_instruction")),
            "valid": [bool(e_hbm.get("valid")), bool(e_tc.get("valid")), bool(e_sfu.get("valid"))]}
    summary["clocks"] = {"sm_mhz": clock.get("sm_mhz"), "mem_mhz": clock.get("mem_mhz"), "reasons": clock.get("reasons")}
    detail = {"hbm": hbm, "tensor": tensor, "gemm_tflops": gemm_tflops, "sfu": sfu, "cache": cache,
              "nonlinear": nonlinear, "telemetry": telemetry, "energy": energy_rows, "clocks": clock}
    return summary, detail


def run_fleet_arms(local: int, world: int, rank: int) -> dict | None:
    """Every rank runs the same arm on its own GPU at the same time, each with its own NVML
    sampler bound to its GPU's UUID (powermodeling_b200.fleet.gpu_arm): HBM read, tcgen05 MMA and
    SFU EX2.  Rank 0 gets the per-GPU rates and their sum."""
    import torch.distributed as dist
    from powermodeling_b200.fleet import gpu_arm
    sms = 148
    arms = {
        "hbm_read_16B_cs_4GiB": (["--workload", "hbm", "--memory-vector-bytes", 16, "--read-cache-policy", "cs",
                                   "--blocks", sms * 8, "--threads", 256, "--working-set-bytes", 4 << 30,
                                   "--iterations", 885, "--batch-launches", 8, "--fixed-batches", 6, *ARM_QUICK],
                                  "throughput_bytes_s", 1e9, "GB/s"),
        "tcgen05_mma_2acc": (["--workload", "tensor", "--blocks", sms, "--threads", 128, "--iterations", 8192,
                              "--tensor-accumulators", 2, "--batch-launches", 4, "--seconds", 2, "--warmup-seconds", 0,
                              "--idle-seconds", 0, "--warmup-batches", 2], "throughput_ops_s", 1e12, "TFLOP/s"),
        "sfu_ex2_148x8": (["--workload", "sfu_ex2", "--grid-mode", "fixed", "--blocks", sms * 8, "--threads", 256,
                           "--sfu-lanes", sms * 8 * 256, "--sfu-chains", 4, "--iterations", 65536, "--batch-launches", 1,
                           "--fixed-batches", 4, *ARM_QUICK], "throughput_ops_s", 1e12, "Tops/s"),
    }
    out = {}
    for name, (args, key, scale, unit) in arms.items():
        dist.barrier()                                  # every GPU starts the arm together
        row = gpu_arm(local, args)
        rows: list = [None] * world
        dist.all_gather_object(rows, {"device": row["device"], "uuid": row["uuid"], "rate": row.get(key),
                                      "sm_mhz": row.get("sm_mhz"), "power_w": row.get("power_w"),
                                      "reasons": row.get("clock_event_reasons")})
        rates = [r["rate"] / scale for r in rows if r["rate"] is not None]
        out[name] = {"unit": unit, "sum": _sig(sum(rates)), "per_gpu": [_sig(v) for v in rates],
                     "gpus_active": len(rates), "sm_mhz": [r["sm_mhz"] for r in rows],
                     "power_w": [_sig(r["power_w"], 4) if r["power_w"] else None for r in rows],
                     "reasons": sorted({x for r in rows for x in (r["reasons"] or [])})}
    return out if rank == 0 else None


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


# Per launch, from one ncu capture of this workload (the committed analysis
# profile summary): warp instructions executed (smsp__inst_executed.sum) and
# DRAM bytes read + written.  The kernels are deterministic for the fixed
# seeds, so the counts are the same on every launch; None where not captured.
NCU_PER_LAUNCH = {
    "analyze_kernel": {"inst": 24_438_012, "dram": 5_002_240},
    "bootstrap_prepare_kernel": {"inst": 7_448_191, "dram": 70_272},
    "bootstrap_kernel<0>": {"inst": 744_303, "dram": 184_320},
}
# Blackwell SM: four schedulers, each issuing one warp instruction per clock.
ISSUE_PER_SM_CLOCK = 4
SMS = 148


def roofline_entry(a_ms, p_ms, f_ms, in_bytes, out_bytes, G, M, packed, peaks, sm_mhz=None):
    """The longest of the three kernels against the bound that limits it.

    The analysis step moves a few MB and does integer/FP64 work per sample
    and per draw, so its roof is instruction issue: warp instructions per
    launch (ncu) over the launch's CUDA-event time, against 4 per SM per
    clock x 148 SMs x the SM clock sampled during the timed steps.  The HBM
    figure of the analysis kernel (input + output bytes over its time) rides
    along for comparison."""
    hbm = peaks.get("hbm_gbs", 6650.0)
    src = "measured" if not peaks.get("fallback") else "fallback"
    times = {"analyze_kernel": a_ms, "bootstrap_prepare_kernel": p_ms, "bootstrap_kernel<0>": f_ms}
    dominant = max(times, key=times.get)
    ms = times[dominant]
    counts = NCU_PER_LAUNCH[dominant]
    clock = sm_mhz or peaks.get("sm_max_mhz", 1965.0)
    issue_peak = ISSUE_PER_SM_CLOCK * SMS * clock * 1e6 / 1e9           # G warp-instructions/s
    entry = {"kernel": dominant, "launch_ms": ms, "traffic": counts["dram"],
             "analyze_kernel_hbm": {"achieved_gbs": (in_bytes + out_bytes) / (a_ms / 1e3) / 1e9, "peak_gbs": hbm,
                                    "frac": (in_bytes + out_bytes) / (a_ms / 1e3) / 1e9 / hbm,
                                    "algorithmic_bytes": in_bytes + out_bytes, "peak_source": src}}
    if counts["inst"] is not None:
        achieved = counts["inst"] / (ms / 1e3) / 1e9
        entry.update(bound="issue", achieved=achieved, peak=issue_peak, unit="G warp-instructions/s",
                     frac=achieved / issue_peak, instructions=counts["inst"],
                     peak_source=f"{ISSUE_PER_SM_CLOCK} warp instructions/clk/SM x {SMS} SMs x {clock:.0f} MHz (sampled)")
    else:
        achieved = (in_bytes + out_bytes) / (a_ms / 1e3) / 1e9
        entry.update(kernel="analyze_kernel", launch_ms=a_ms, bound="hbm", achieved=achieved, peak=hbm, unit="GB/s",
                     frac=achieved / hbm, traffic=NCU_PER_LAUNCH["analyze_kernel"]["dram"], peak_source=src)
    return entry


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
    """The reference's CPU analysis restated (oracle), all host cores, on the same workload.

    One step = the 64-point sweep of one GPU's share (256 trials, 64 groups of 4
    at B = 10 000) from the record dicts: the trials are analysed and every
    group's medians and intervals computed by processes over groups on every
    host core (the records of each group are sent to its process inside the
    step, as summarize(records) receives them)."""
    from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
    records = make_sweep(SweepShape(points=POINTS, repeats=REPEATS), seed=0)
    pol = dict(__import__("oracle.analysis_oracle", fromlist=["DEFAULT_POLICY"]).DEFAULT_POLICY, **ANALYSIS_POLICY)
    cores = os.cpu_count() or 1
    jobs = [(records[i * REPEATS:(i + 1) * REPEATS], 1000003 + i, pol, RESAMPLES) for i in range(POINTS)]
    samples = sum(len(ph.get("samples", [])) for r in records for ph in (r.get("phases") or {}).values())
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(args.warmup):
            pool.map(_oracle_group, jobs, chunksize=1)
        times, resamples = [], 0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            resamples += sum(pool.map(_oracle_group, jobs, chunksize=1))
            times.append(time.perf_counter() - t0)
    step_s = sum(times) / len(times)
    value = resamples / sum(times)
    world = max(1, args.gpus)
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "resamples/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "points": POINTS * world, "points_per_gpu": POINTS, "repeats": REPEATS,
                       "trials": POINTS * REPEATS * world, "groups": POINTS * world, "resamples": RESAMPLES,
                       "samples": samples, "l2": "n/a (host)",
                       "parallelism": f"processes over groups, {cores} host cores"},
            "cpu_baseline": {"value": value, "unit": "resamples/s", "cores": cores, "kind": "port",
                             "sample": f"each step the {POINTS}-point sweep of one GPU's share "
                                       f"({POINTS * REPEATS} trials, {POINTS} groups) from the record dicts, "
                                       f"processes over groups on {cores} cores"},
            "e2e": {"value": value, "unit": "resamples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--exchange", choices=("peer", "nccl"), default="peer",
                        help="N>1: group results stored into rank 0 by the bootstrap kernel over NVLink, or all-gathered by NCCL")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--scaling", choices=("weak", "strong"), default="weak",
                        help="weak: 64 points per GPU; strong: one 64-point sweep split over the GPUs by points")
    parser.add_argument("--no-arms", action="store_true", help="skip the HBM/tensor/GEMM/SFU arm measurements")
    parser.add_argument("--no-energy", action="store_true", help="skip the captured 10 s energy trials of the arms")
    parser.add_argument("--arms-detail", help="also write every arm row to this JSON file")
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
        # The ranks share the host's cores: each rank's record packer and staging pool take
        # their share instead of all of them (the variables are read once, at first use).
        share = max(1, (len(os.sched_getaffinity(0)) or 1) // int(os.environ.get("LOCAL_WORLD_SIZE", world)))
        os.environ.setdefault("PM_PACK_THREADS", str(min(16, share)))
        os.environ.setdefault("PM_HOST_THREADS", str(max(1, min(3, share - 1))))
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        torch.set_num_threads(min(torch.get_num_threads(), share))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        line = run_b200(args, rank, world)
        if line is not None:
            print(json.dumps(compact(line)), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
