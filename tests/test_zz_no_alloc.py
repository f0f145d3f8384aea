"""The allocation-free bootstrap entry point against the allocating one (GPU).

pm_group_bootstrap_device_static serves callers that cannot let a library
call cudaMalloc; it keeps its index streams in a fixed array compiled into
libpmb200.  This file is collected last so that a failure here, under -x,
comes after every other test has run.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from powermodeling_b200 import _native as N
from powermodeling_b200.analysis import bootstrap_groups

pytestmark = pytest.mark.gpu


def _groups(rng, sizes, metrics):
    rows = sum(sizes)
    values = rng.normal(100.0, 15.0, size=(rows, metrics))
    values[rng.random(size=values.shape) < 0.05] = np.nan          # some None entries
    members = []
    start = 0
    for size in sizes:
        members.append(list(range(start, start + size)))
        start += size
    seeds = [int(x) for x in rng.integers(0, 2 ** 63, size=len(sizes), dtype=np.uint64)]
    return values, members, seeds


def _static_call(torch, lib, values, members, seeds, resamples):
    G, M = len(members), values.shape[1]
    offsets = np.zeros(G + 1, dtype=np.int32)
    np.cumsum([len(m) for m in members], out=offsets[1:])
    rows = np.concatenate([np.asarray(m, dtype=np.int32) for m in members])
    d_values = torch.from_numpy(np.ascontiguousarray(values)).cuda()
    d_offsets, d_rows = torch.from_numpy(offsets).cuda(), torch.from_numpy(rows).cuda()
    d_seeds = torch.from_numpy(np.asarray(seeds, dtype=np.uint64).view(np.int64)).cuda()
    med, lo, hi = (torch.empty(G * M, dtype=torch.float64, device="cuda") for _ in range(3))
    job = N.BootstrapJob(G, M, int(rows.size), values.shape[0], resamples, max(len(m) for m in members),
                         d_values.data_ptr(), d_offsets.data_ptr(), d_rows.data_ptr(), None, d_seeds.data_ptr(),
                         med.data_ptr(), lo.data_ptr(), hi.data_ptr())
    stream = torch.cuda.current_stream()
    N.check(lib.pm_group_bootstrap_device_static(job, C.c_void_p(stream.cuda_stream)), "pm_group_bootstrap_device_static")
    stream.synchronize()
    return [t.cpu().numpy().reshape(G, M) for t in (med, lo, hi)]


def test_static_bootstrap_matches_allocating_entry_point_twice():
    import torch
    lib = N.library()
    if lib.pm_device_count() < 1:
        pytest.fail("GPU test ran without a visible CUDA device")
    lib.pm_group_bootstrap_device_static.argtypes = [C.POINTER(N.BootstrapJob), C.c_void_p]
    lib.pm_bootstrap_static_scratch_capacity.restype = C.c_size_t
    assert lib.pm_bootstrap_static_scratch_capacity() == 32 << 20
    rng = np.random.default_rng(20261201)
    # Every group's index stream in the fixed array (the streamed prepare pass); the last job's streams
    # do not fit, so its groups of up to seven members are drawn and counted in one pass instead.
    many = tuple(3 + i % 5 for i in range(3000))
    assert 3000 * 10000 * 7 > 32 << 20 > 3000 * 1716 * 4
    for sizes, resamples, metrics in (((9, 12, 5, 20), 10000, 47), ((8, 3, 16), 1000, 47), (many, 10000, 3)):
        values, members, seeds = _groups(rng, sizes, metrics)
        expected = bootstrap_groups(values, members, seeds, resamples)          # allocating host entry point
        got = _static_call(torch, lib, values, members, seeds, resamples)
        for e, g in zip(expected, got):
            assert np.array_equal(np.isnan(e), np.isnan(g))
            assert np.array_equal(np.nan_to_num(e), np.nan_to_num(g))        # the same kernel: bit-exact


def test_static_bootstrap_rejects_jobs_beyond_its_array():
    lib = N.library()
    lib.pm_group_bootstrap_device_static.argtypes = [C.POINTER(N.BootstrapJob), C.c_void_p]
    dummy = C.c_double(0.0)
    # 64 groups of up to 64 members at 10 000 resamples: 41 MB of index streams, rejected before any launch.
    assert 64 * 10000 * 64 > 32 << 20
    job = N.BootstrapJob(64, 1, 64 * 64, 64 * 64, 10000, 64, C.addressof(dummy), C.addressof(dummy), None, None,
                         C.addressof(dummy), C.addressof(dummy), C.addressof(dummy), C.addressof(dummy))
    rc = lib.pm_group_bootstrap_device_static(job, None)
    assert rc == -4 and "fixed array holds" in N.last_error()
