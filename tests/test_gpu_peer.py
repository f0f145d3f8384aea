"""The NVLink peer-memory exchanges of the sharded step (include/pmb200_peer.h).

Two GPUs: rows and group results stored into every rank by the analysis and
bootstrap kernels equal, bit for bit, an NCCL all-gather of the same local
outputs, over several epochs, with the groups split evenly over the ranks
and with one rank owning a group fewer (its last slot is never written).  One GPU: the arrival wait ends on its own
limit when a flag is never raised, reports it, and leaves the context usable.
"""
from __future__ import annotations

import ctypes as C
import json
import multiprocessing as mp
import os
import socket
import tempfile

import pytest

pytestmark = pytest.mark.gpu

POINTS, REPEATS, STEPS = 4, 4, 3


def _worker(rank, world, port, out_path, uneven=False):
    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    result = {}
    try:
        import bench
        from powermodeling_b200 import _native as N
        from powermodeling_b200 import analysis as A
        from powermodeling_b200.peer import PeerExchange
        from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep
        lib = N.library()
        records = make_sweep(SweepShape(points=POINTS, repeats=REPEATS), seed=11 + rank, first_point=rank * POINTS)
        packed, _, _ = A.prepare(records)
        trials, keep, _ = bench.device_arrays(packed, torch)
        n, M = packed.n_trials, N.layout("PM_M_COUNT")
        PO, TO = N.layout("PM_PO_COUNT"), N.layout("PM_TO_COUNT")
        out = {"phase_out": torch.empty(n * 5 * PO, dtype=torch.float64, device="cuda"),
               "phase_flags": torch.empty(n * 5, dtype=torch.int32, device="cuda"),
               "trial_out": torch.empty(n * TO, dtype=torch.float64, device="cuda"),
               "issue_bits": torch.empty(n * 4, dtype=torch.int64, device="cuda"),
               "metrics": torch.empty(n * M, dtype=torch.float64, device="cuda"),
               "valid": torch.empty(n, dtype=torch.uint8, device="cuda")}
        results = N.TrialResults(*(out[k].data_ptr() for k in ("phase_out", "phase_flags", "trial_out", "issue_bits",
                                                                "metrics", "valid")))
        policy = A.AnalysisPolicy(**ANALYSIS_POLICY).native()
        # groups: every point's repeats (global rows), owned round robin
        G = world * POINTS - (1 if uneven else 0)
        members = [[(g // POINTS) * n + (g % POINTS) * REPEATS + k for k in range(REPEATS)] for g in range(G)]
        mine = [g for g in range(G) if g % world == rank]
        per_rank = -(-G // world)
        px = PeerExchange(rank, world, n, M, per_rank)
        offsets = np.zeros(len(mine) + 1, dtype=np.int32)
        np.cumsum([len(members[g]) for g in mine], out=offsets[1:])
        rows = np.concatenate([np.asarray(members[g], dtype=np.int32) for g in mine])
        d_off, d_rows = torch.from_numpy(offsets).cuda(), torch.from_numpy(rows).cuda()
        d_seeds = torch.from_numpy((np.asarray(mine, dtype=np.uint64) * 7919 + 17).view(np.int64)).cuda()
        group_out = torch.full((3, per_rank, M), float("nan"), dtype=torch.float64, device="cuda")
        job = N.BootstrapJob(len(mine), M, int(rows.size), world * n, 1000, REPEATS, px.metrics_ptr, d_off.data_ptr(),
                             d_rows.data_ptr(), px.valid_ptr, d_seeds.data_ptr(), group_out[0].data_ptr(),
                             group_out[1].data_ptr(), group_out[2].data_ptr())
        a_scr = lib.pm_analyze_scratch_bytes(n, packed.max_phase_samples)
        b_scr = lib.pm_bootstrap_scratch_bytes(len(mine), REPEATS, 1000)
        scratch = torch.empty(max(1, a_scr + b_scr), dtype=torch.uint8, device="cuda")
        stream = torch.cuda.current_stream()
        sptr = C.c_void_p(stream.cuda_stream)
        boot = C.c_void_p(scratch.data_ptr() + a_scr)
        for _ in range(STEPS):
            px.next_epoch()
            N.check(lib.pm_analyze_trials_device_exchange(trials, policy, results, C.c_void_p(scratch.data_ptr()), a_scr,
                                                          C.byref(px.rows), sptr), "analyze + rows")
            px.wait_rows(stream.cuda_stream)
            N.check(lib.pm_bootstrap_prepare_device(job, boot, b_scr, sptr), "prepare")
            N.check(lib.pm_bootstrap_finish_device_exchange(job, boot, b_scr, C.byref(px.groups), sptr), "finish + groups")
            px.wait_groups(stream.cuda_stream)
        px.check()
        want_rows = torch.empty(world * n * M, dtype=torch.float64, device="cuda")
        want_valid = torch.empty(world * n, dtype=torch.uint8, device="cuda")
        want_groups = torch.empty((world, 3, per_rank, M), dtype=torch.float64, device="cuda")
        dist.all_gather_into_tensor(want_rows, out["metrics"])
        dist.all_gather_into_tensor(want_valid, out["valid"])
        dist.all_gather_into_tensor(want_groups, group_out)
        torch.cuda.synchronize()
        got_rows, got_valid, got_groups = px.view("metrics"), px.view("valid"), px.view("groups")
        # each rank's owned slots (a rank with fewer groups leaves its last slot unwritten)
        owned = [len([g for g in range(G) if g % world == r]) for r in range(world)]
        same_groups = all(torch.equal(got_groups[r, :, :owned[r]].reshape(-1).view(torch.int64),
                                      want_groups[r, :, :owned[r]].reshape(-1).view(torch.int64)) for r in range(world))
        result = {"rows": bool(torch.equal(got_rows.reshape(-1).view(torch.int64), want_rows.view(torch.int64))),
                  "valid": bool(torch.equal(got_valid, want_valid)),
                  "groups": bool(same_groups),
                  "groups_finite": int(torch.isfinite(want_groups[:, 1]).sum().item()),
                  "epoch": int(px.rows.epoch)}
        px.close()
    finally:
        with open(f"{out_path}.{rank}", "w") as f:
            json.dump(result, f)
        dist.destroy_process_group()


@pytest.mark.parametrize("uneven", [False, True], ids=["even", "one-group-fewer"])
def test_two_gpu_peer_exchange_equals_all_gather(gpu_ready, uneven):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    os.environ.update(env)
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "peer")
        procs = [ctx.Process(target=_worker, args=(r, world, port, out, uneven)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        for r in range(world):
            with open(f"{out}.{r}") as f:
                got = json.load(f)
            assert got == {"rows": True, "valid": True, "groups": True, "groups_finite": got["groups_finite"],
                           "epoch": STEPS}, got
            assert got["groups_finite"] > 0


def test_arrival_wait_ends_on_its_limit(gpu_ready):
    import time
    import torch
    from powermodeling_b200 import _native as N
    lib = N.library()
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")        # nothing ever raises them
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    t0 = time.perf_counter()
    N.check(lib.pm_peer_wait_device(C.c_void_p(flags.data_ptr()), 2, 1, 50, C.c_void_p(error.data_ptr()),
                                    C.c_void_p(stream.cuda_stream)), "wait")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(error.item()) == 1 and 0.04 < waited < 5.0
    # the context is still usable, and raised flags pass at once
    error.zero_()
    flags.fill_(1)
    N.check(lib.pm_peer_wait_device(C.c_void_p(flags.data_ptr()), 2, 1, 50, C.c_void_p(error.data_ptr()),
                                    C.c_void_p(stream.cuda_stream)), "wait")
    torch.cuda.synchronize()
    assert int(error.item()) == 0
    assert float((torch.arange(4, device="cuda") * 2).sum().item()) == 12.0
