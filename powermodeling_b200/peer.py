"""The sharded summarize's exchanges over NVLink peer memory (include/pmb200_peer.h).

One process per GPU.  ``PeerExchange`` allocates this rank's gathered
buffers (metric rows and valid flags of every rank's trials, when rows move
at all; medians and interval ends of every rank's groups; arrival flags and
counters; the start-line flags), swaps their CUDA IPC handles over a torch
process group, opens the other ranks' buffers and fills the
``pm_peer_rows`` / ``pm_peer_groups`` descriptors that
``pm_analyze_trials_device_exchange`` and
``pm_bootstrap_finish_device_exchange`` take.  The kernels store straight
into the receiving ranks' buffers; ``wait_rows`` / ``wait_groups`` hold a
stream until every rank's launch has delivered, each wait bounded (an
expired wait raises here, after the stream drains); ``gate`` starts all
ranks' following work together on their GPUs.

With ``rows_per_rank=0`` no rows move: every group is bootstrapped on the
rank that analysed its members, and only the group results travel, to every
rank (``root=-1``) or to one rank (a gather).
"""
from __future__ import annotations

import ctypes as C

from . import _native as N


class PeerExchangeError(RuntimeError):
    """The exchange could not be set up; every rank of the group raises it together."""


class PeerExchange:
    """Gathered row and group buffers of one rank, shared with every other rank.

    rows_per_rank: trials each rank analyses (rank r's trial t is global row
    r * rows_per_rank + t), 0 when no rows are exchanged; groups_per_rank: the
    group stride of the gathered group buffer ([world][3][groups_per_rank][n_metrics]);
    root: -1 to deliver group results to every rank, else the one rank that
    receives them."""

    def __init__(self, rank: int, world: int, rows_per_rank: int, n_metrics: int, groups_per_rank: int,
                 group=None, timeout_ms: int = 5000, root: int = -1):
        import torch
        import torch.distributed as dist
        if not 1 <= world <= N.MAX_RANKS:
            raise ValueError(f"world size must be 1..{N.MAX_RANKS}")
        if not -1 <= root < world:
            raise ValueError("root must be -1 or a rank")
        self.lib = N.library()
        self.rank, self.world, self.timeout_ms, self.root = rank, world, timeout_ms, root
        self.rows_per_rank, self.n_metrics, self.groups_per_rank = rows_per_rank, n_metrics, groups_per_rank
        total_rows = world * rows_per_rank
        sizes = {"groups": world * 3 * max(1, groups_per_rank) * n_metrics * 8, "group_flags": (world + 1) * 4,
                 "gate": world * 4}
        if rows_per_rank > 0:
            sizes.update(metrics=total_rows * n_metrics * 8, valid=total_rows, row_flags=(world + 1) * 4)
        names = list(sizes)
        # Every rank takes both collectives below, whatever failed locally, so a
        # failure on one rank becomes the same PeerExchangeError on all of them.
        self.own, self.opened, handles, failure = {}, [], [], None
        try:
            for name in names:
                ptr, handle = C.c_void_p(), N.PeerHandle()
                N.check(self.lib.pm_peer_alloc(sizes[name], C.byref(ptr), C.byref(handle)), "pm_peer_alloc")
                self.own[name] = ptr.value
                handles.append(bytes(handle.bytes))
        except N.NativeError as exc:
            failure = str(exc)
        everyone: list = [None] * world
        dist.all_gather_object(everyone, None if failure else handles, group=group)
        missing = [r for r, h in enumerate(everyone) if h is None]
        if missing:
            self._release()
            raise PeerExchangeError(f"peer buffers could not be allocated on rank(s) {missing}"
                                    + (f": {failure}" if failure else ""))
        per_rank: list[dict] = []
        try:
            for r in range(world):
                if r == rank:
                    per_rank.append(dict(self.own))
                    continue
                ptrs = {}
                for name, raw in zip(names, everyone[r]):
                    h, q = N.PeerHandle(), C.c_void_p()
                    C.memmove(h.bytes, raw, 64)
                    N.check(self.lib.pm_peer_open(C.byref(h), C.byref(q)), "pm_peer_open")
                    self.opened.append(q.value)
                    ptrs[name] = q.value
                per_rank.append(ptrs)
        except N.NativeError as exc:
            failure = str(exc)
        opened = torch.tensor([0 if failure else 1], dtype=torch.int32, device="cuda")
        dist.all_reduce(opened, op=dist.ReduceOp.MIN, group=group)
        if not int(opened.item()):
            self._release()
            raise PeerExchangeError("another rank's buffers could not be opened"
                                    + (f" on rank {rank}: {failure}" if failure else " (on another rank)"))
        self.rows, self.groups = N.PeerRows(), N.PeerGroups()
        self.rows.n_ranks, self.rows.rank, self.rows.row_offset, self.rows.epoch = world, rank, rank * rows_per_rank, 0
        self.groups.n_ranks, self.groups.rank, self.groups.per_rank, self.groups.epoch = world, rank, groups_per_rank, 0
        self.groups.root = root
        self.gate_flags = (C.c_void_p * world)()
        for r, ptrs in enumerate(per_rank):
            if rows_per_rank > 0:
                self.rows.metrics[r], self.rows.valid[r], self.rows.flags[r] = ptrs["metrics"], ptrs["valid"], ptrs["row_flags"]
            self.groups.out[r], self.groups.flags[r] = ptrs["groups"], ptrs["group_flags"]
            self.gate_flags[r] = ptrs["gate"]
        if rows_per_rank > 0:
            self.rows.done = self.own["row_flags"] + world * 4
        self.groups.done = self.own["group_flags"] + world * 4
        self.gate_epoch = 0
        self.error = torch.zeros(1, dtype=torch.int32, device="cuda")
        self._group = group

    # gathered buffers of this rank (device pointers) ----------------------------------------------
    @property
    def metrics_ptr(self) -> int:
        return self.own["metrics"]

    @property
    def valid_ptr(self) -> int:
        return self.own["valid"]

    @property
    def groups_ptr(self) -> int:
        return self.own["groups"]

    def view(self, which: str):
        """A torch tensor over this rank's gathered 'metrics', 'valid' or 'groups' buffer (no copy)."""
        import torch
        total = self.world * self.rows_per_rank
        shape, typestr, ptr = {
            "metrics": ((total, self.n_metrics), "<f8", self.own.get("metrics")),
            "valid": ((total,), "|u1", self.own.get("valid")),
            "groups": ((self.world, 3, max(1, self.groups_per_rank), self.n_metrics), "<f8", self.own["groups"]),
        }[which]

        class _View:
            __cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                        "strides": None}
        return torch.as_tensor(_View(), device="cuda")

    # one step -----------------------------------------------------------------------------------
    def next_epoch(self) -> None:
        """Advance both exchanges to the next step (every launch uses a new epoch)."""
        self.rows.epoch += 1
        self.groups.epoch += 1

    def wait_rows(self, stream_ptr: int) -> None:
        N.check(self.lib.pm_peer_wait_device(C.c_void_p(self.own["row_flags"]), self.world, self.rows.epoch,
                                             self.timeout_ms, C.c_void_p(self.error.data_ptr()), C.c_void_p(stream_ptr)),
                "row arrival wait")

    def wait_groups(self, stream_ptr: int) -> None:
        """Hold the stream until every rank's groups of this epoch are here (receiving ranks only)."""
        N.check(self.lib.pm_peer_wait_device(C.c_void_p(self.own["group_flags"]), self.world, self.groups.epoch,
                                             self.timeout_ms, C.c_void_p(self.error.data_ptr()), C.c_void_p(stream_ptr)),
                "group arrival wait")

    def gate(self, stream_ptr: int) -> None:
        """Start line: work this rank enqueues after it starts on its GPU once every rank has reached it."""
        self.gate_epoch += 1
        N.check(self.lib.pm_peer_gate_device(self.gate_flags, self.world, self.rank, self.gate_epoch, self.timeout_ms,
                                             C.c_void_p(self.error.data_ptr()), C.c_void_p(stream_ptr)), "start gate")

    def check(self) -> None:
        """Raise if any wait expired (synchronizes the device)."""
        import torch
        torch.cuda.synchronize()
        if int(self.error.item()):
            raise N.NativeError("a rank's rows or groups did not arrive within the wait limit")

    def close(self) -> None:
        """Release the buffers (a barrier first: no rank may still be storing into them)."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=self._group)
        self._release(check=True)

    def _release(self, check: bool = False) -> None:
        for q in self.opened:
            rc = self.lib.pm_peer_close(C.c_void_p(q))
            if check:
                N.check(rc, "pm_peer_close")
        for q in self.own.values():
            rc = self.lib.pm_peer_free(C.c_void_p(q))
            if check:
                N.check(rc, "pm_peer_free")
        self.opened, self.own = [], {}
