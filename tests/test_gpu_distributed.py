"""Sharded summarize over NCCL on two GPUs equals the one-GPU summarize (skipped with fewer GPUs)."""
from __future__ import annotations

import multiprocessing as mp
import os
import pickle
import socket
import tempfile

import pytest

pytestmark = pytest.mark.gpu


def _records(rank: int, world: int):
    from powermodeling_b200.synthetic import SweepShape, make_sweep
    records = make_sweep(SweepShape(points=6, repeats=4), seed=5)
    mine = [r for i, r in enumerate(records) if (i // 4) % world == rank]   # whole points per rank
    if rank == world - 1:
        mine.append(dict(records[0]))                                        # a duplicate across ranks
    return mine


def _worker(rank, world, port, out_path):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from powermodeling_b200.distributed import summarize_sharded
        from powermodeling_b200.synthetic import ANALYSIS_POLICY
        summary = summarize_sharded(_records(rank, world), policy=ANALYSIS_POLICY, resamples=1000)
        with open(f"{out_path}.{rank}", "wb") as f:
            pickle.dump(summary, f)
    finally:
        dist.destroy_process_group()


def same(a, b) -> bool:
    """Deep equality with NaN equal to NaN (objects that crossed a process boundary pickle differently)."""
    if isinstance(a, float) and isinstance(b, float):
        return a == b or (a != a and b != b)
    if isinstance(a, dict) and isinstance(b, dict):
        return a.keys() == b.keys() and all(same(a[k], b[k]) for k in a)
    if isinstance(a, (list, tuple)) and isinstance(b, (list, tuple)):
        return len(a) == len(b) and all(same(x, y) for x, y in zip(a, b))
    return type(a) is type(b) and a == b


def test_two_gpu_sharded_summary_equals_single_gpu(gpu_ready):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from powermodeling_b200.analysis import summarize
    from powermodeling_b200.synthetic import ANALYSIS_POLICY
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "summary")
        procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
        results = []
        for r in range(world):
            with open(f"{out}.{r}", "rb") as f:
                results.append(pickle.load(f))
    ordered = [rec for r in range(world) for rec in _records(r, world)]
    expected = summarize(ordered, policy=ANALYSIS_POLICY, resamples=1000)
    for got in results:
        assert [g["group_id"] for g in got["groups"]] == [g["group_id"] for g in expected["groups"]]
        assert same(got["groups"], expected["groups"])
        assert same(got["trials"], expected["trials"])
        assert got["duplicate_trial_ids_ignored"] == expected["duplicate_trial_ids_ignored"]
        assert [t["trial_id"] for t in got["trials"]] == [t["trial_id"] for t in expected["trials"]]
