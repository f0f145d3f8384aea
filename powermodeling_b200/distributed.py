"""One sweep summarized across ranks: trials and groups sharded, two exchanges.

``summarize_sharded`` is ``analysis.summarize`` over the records of all
ranks taken in rank order, computed with one process per GPU:

1. trial ids are gathered so duplicates are dropped in the global order
   (analysis.py:1408-1416);
2. each rank analyses its own records (one ``analyze_kernel`` launch);
3. exchange one — every rank receives every trial record and metric row
   (rows as one tensor all-gather over the process group's backend, NCCL on
   GPUs);
4. the groups (key order, valid members, sha256 seeds) are formed
   identically on every rank, and rank r bootstraps groups r, r + world, ...
   (one ``bootstrap_kernel`` launch over the gathered rows);
5. exchange two — the group medians and interval bounds are all-gathered and
   every rank assembles the same summary.

Each group's intervals are computed whole by one rank from the group's own
MT19937 stream, so the result equals the single-process summary exactly.
"""
from __future__ import annotations

from typing import Any, Iterable, Mapping

import numpy as np

from . import analysis as A


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of ``n`` items for ``rank``; the first n % world ranks take one more."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def owned_groups(n_groups: int, world: int, rank: int) -> list[int]:
    """Groups bootstrapped by ``rank``: round robin, so group sizes even out across ranks."""
    return list(range(rank, n_groups, world))


def _tensor_device(group):
    import torch
    import torch.distributed as dist
    return torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")


def _all_gather_rows(local: np.ndarray, counts: list[int], group) -> np.ndarray:
    """Concatenation of every rank's rows (rank order) through one tensor all-gather."""
    import torch
    import torch.distributed as dist
    world = len(counts)
    width = local.shape[1]
    most = max(counts) if counts else 0
    device = _tensor_device(group)
    padded = torch.full((max(most, 1), width), float("nan"), dtype=torch.float64, device=device)
    if local.shape[0]:
        padded[:local.shape[0]] = torch.from_numpy(np.ascontiguousarray(local)).to(device)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return np.concatenate([parts[r][:counts[r]].cpu().numpy() for r in range(world)], axis=0) if counts else local


def _all_gather_groups(n_groups: int, width: int, mine: list[int], outputs, world: int, group):
    """Full (n_groups x width) medians, lows and highs from each rank's owned groups."""
    import torch
    import torch.distributed as dist
    device = _tensor_device(group)
    per_rank = -(-n_groups // world) if n_groups else 0
    block = torch.full((3, max(per_rank, 1), width), float("nan"), dtype=torch.float64, device=device)
    for k, array in enumerate(outputs):
        if len(mine):
            block[k, :len(mine)] = torch.from_numpy(np.ascontiguousarray(array)).to(device)
    parts = [torch.empty_like(block) for _ in range(world)]
    dist.all_gather(parts, block, group=group)
    med, lo, hi = (np.full((n_groups, width), np.nan) for _ in range(3))
    for r in range(world):
        owned = owned_groups(n_groups, world, r)
        host = parts[r].cpu().numpy()
        for j, g in enumerate(owned):
            med[g], lo[g], hi[g] = host[0, j], host[1, j], host[2, j]
    return med, lo, hi


def summarize_sharded(records: Iterable[Mapping[str, Any]], throughput_fraction: float = 0.95,
                      policy: A.AnalysisPolicy | Mapping[str, Any] | None = None, min_repeats: int = 3,
                      hbm_bandwidth_fraction: float = 0.80, resamples: int = A.DEFAULT_RESAMPLES,
                      group=None, plan=None, evaluation_policy=None, plan_validator=None) -> dict[str, Any]:
    """``summarize`` of all ranks' records (rank order); each rank passes its own and gets the whole summary.
    The evaluation's display traces are gathered as trace points, not whole records."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    hbm_bandwidth_fraction = A.check_summary_arguments(throughput_fraction, min_repeats, hbm_bandwidth_fraction)
    policy = A._policy(policy)
    records = list(records)
    ids: list = [None] * world
    dist.all_gather_object(ids, [r.get("trial_id") for r in records], group=group)
    seen, duplicates, keep = set(), [], []
    for r, part in enumerate(ids):
        for i, trial_id in enumerate(part):
            if trial_id is not None and trial_id in seen:
                duplicates.append(trial_id)
                continue
            if trial_id is not None:
                seen.add(trial_id)
            if r == rank:
                keep.append(i)
    local_trials, local_rows = A.analyze_rows([records[i] for i in keep], policy, hbm_bandwidth_fraction)
    parts: list = [None] * world
    dist.all_gather_object(parts, local_trials, group=group)
    trials = [t for part in parts for t in part]
    counts = [len(part) for part in parts]
    width = len(A.METRICS) + len(A.SENSOR_FIELDS)
    rows = _all_gather_rows(local_rows.reshape(len(local_trials), width), counts, group)
    groups, members, seeds, group_indices = A.group_structure(trials, min_repeats)
    mine = owned_groups(len(groups), world, rank)
    if mine:
        outputs = A.bootstrap_groups(rows, [members[g] for g in mine], [seeds[g] for g in mine], resamples)
    else:
        outputs = tuple(np.zeros((0, width)) for _ in range(3))
    med, lo, hi = _all_gather_groups(len(groups), width, mine, outputs, world, group)
    A.finish_groups(groups, trials, members, group_indices, med, lo, hi, hbm_bandwidth_fraction, min_repeats)
    summary = A.summary_record(trials, groups, duplicates, throughput_fraction, hbm_bandwidth_fraction, min_repeats,
                               resamples, policy)
    from .evaluation import evaluate, trace_points
    shards: list = [None] * world
    dist.all_gather_object(shards, [(r.get("trial_id"), trace_points(r)) for r in records], group=group)
    traces = {trial_id: points for shard in shards for trial_id, points in shard}   # the last record of an id wins
    summary["evaluation"] = evaluate(summary, plan=plan, policy=evaluation_policy, plan_validator=plan_validator,
                                     traces=traces)
    return summary
