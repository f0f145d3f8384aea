"""pm_analyze_sweep_device (the whole sweep on device buffers in one call) against the
separate entry points: the same trial results and group intervals, bit for bit."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from powermodeling_b200 import _native as N
from powermodeling_b200 import analysis as A
from powermodeling_b200.synthetic import ANALYSIS_POLICY, SweepShape, make_sweep

pytestmark = pytest.mark.gpu

B = 10000


def _device_sweep(torch, points: int, seed: int):
    records = make_sweep(SweepShape(points=points, repeats=4), seed=seed)
    policy = A.AnalysisPolicy(**ANALYSIS_POLICY)
    packed, _, _ = A.prepare(records)
    trials = A.analyze_trials(records, policy)
    buckets: dict[str, list[int]] = {}
    for i, t in enumerate(trials):
        buckets.setdefault(A.group_key(t), []).append(i)
    keys = sorted(buckets)
    members, seeds = [buckets[k] for k in keys], [A.group_seed(k) for k in keys]
    dev = {}
    t = N.Trials()
    t.n_trials, t.max_phase_samples, t.n_samples, t.n_epochs = packed.n_trials, packed.max_phase_samples, packed.n_samples, packed.n_epochs
    t.broadcast_columns = packed.broadcast
    for name, _, _ in N.TRIAL_ARRAYS + N.EPOCH_ARRAYS + N.TAIL_ARRAYS:
        a = packed.arrays[name]
        dev[name] = torch.from_numpy(a.copy()).cuda() if a.size else torch.empty(1, dtype=torch.uint8, device="cuda")
        setattr(t, name, dev[name].data_ptr())
    return packed, policy.native(), t, dev, members, seeds


def _outputs(torch, n, G, M):
    PO, TO = N.layout("PM_PO_COUNT"), N.layout("PM_TO_COUNT")
    out = {"phase_out": torch.empty(n * 5 * PO, dtype=torch.float64, device="cuda"),
           "phase_flags": torch.empty(n * 5, dtype=torch.int32, device="cuda"),
           "trial_out": torch.empty(n * TO, dtype=torch.float64, device="cuda"),
           "issue_bits": torch.empty(n * 4, dtype=torch.int64, device="cuda"),
           "metrics": torch.empty(n * M, dtype=torch.float64, device="cuda"),
           "valid": torch.empty(n, dtype=torch.uint8, device="cuda"),
           "groups": torch.full((3, max(G, 1), M), float("nan"), dtype=torch.float64, device="cuda")}
    res = N.TrialResults(*(out[k].data_ptr() for k in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid")))
    return out, res


def test_sweep_device_equals_separate_entry_points(gpu_ready):
    torch = pytest.importorskip("torch")
    lib = N.library()
    M = len(A.METRICS)
    packed, pol, t, _dev, members, seeds = _device_sweep(torch, 16, 5)
    n, G = packed.n_trials, len(members)
    offsets = np.zeros(G + 1, dtype=np.int32)
    np.cumsum([len(m) for m in members], out=offsets[1:])
    rows = np.concatenate([np.asarray(m, dtype=np.int32) for m in members])
    d_off, d_rows = torch.from_numpy(offsets).cuda(), torch.from_numpy(rows).cuda()
    d_seeds = torch.from_numpy(np.asarray(seeds, dtype=np.uint64).view(np.int64)).cuda()
    max_members = max(len(m) for m in members)

    def job_for(out):
        g = out["groups"]
        return N.BootstrapJob(G, M, int(rows.size), n, B, max_members, out["metrics"].data_ptr(), d_off.data_ptr(),
                              d_rows.data_ptr(), out["valid"].data_ptr(), d_seeds.data_ptr(),
                              g[0].data_ptr(), g[1].data_ptr(), g[2].data_ptr())

    # the separate calls
    ref, ref_res = _outputs(torch, n, G, M)
    ref_job = job_for(ref)
    a_scr = lib.pm_analyze_scratch_bytes(n, packed.max_phase_samples)
    b_scr = lib.pm_bootstrap_scratch_bytes(G, max_members, B)
    b_off = (a_scr + 255) // 256 * 256                      # the bootstrap's scratch on a 256-byte boundary
    scratch = torch.empty(b_off + b_scr, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    N.check(lib.pm_analyze_trials_device(t, pol, ref_res, C.c_void_p(scratch.data_ptr()), a_scr, C.c_void_p(s)), "analyze")
    N.check(lib.pm_group_bootstrap_device(ref_job, C.c_void_p(scratch.data_ptr() + b_off), b_scr, C.c_void_p(s)),
            "bootstrap")
    torch.cuda.synchronize()

    # the one call, on the current stream and on the legacy default stream, three times each
    need = lib.pm_analyze_sweep_scratch_bytes(n, packed.max_phase_samples, G, max_members, B)
    assert need >= b_scr
    sweep_scratch = torch.empty(need, dtype=torch.uint8, device="cuda")
    for stream in (C.c_void_p(s), None, C.c_void_p(s)):
        got, got_res = _outputs(torch, n, G, M)
        N.check(lib.pm_analyze_sweep_device(t, pol, got_res, job_for(got), C.c_void_p(sweep_scratch.data_ptr()), need, None,
                                            stream), "pm_analyze_sweep_device")
        torch.cuda.synchronize()
        for key in ("phase_out", "phase_flags", "trial_out", "issue_bits", "metrics", "valid", "groups"):
            a, b = ref[key].cpu().numpy(), got[key].cpu().numpy()
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), key
    assert int(ref["valid"].sum().item()) == n
    assert np.isfinite(ref["groups"][1].cpu().numpy()).any()


def test_sweep_device_rejects_short_scratch(gpu_ready):
    torch = pytest.importorskip("torch")
    lib = N.library()
    M = len(A.METRICS)
    packed, pol, t, _dev, members, seeds = _device_sweep(torch, 2, 1)
    n, G = packed.n_trials, len(members)
    out, res = _outputs(torch, n, G, M)
    d_off = torch.tensor([0, 4, 8][:G + 1], dtype=torch.int32, device="cuda")
    d_seeds = torch.from_numpy(np.asarray(seeds, dtype=np.uint64).view(np.int64)).cuda()
    g = out["groups"]
    job = N.BootstrapJob(G, M, 4 * G, n, B, 4, out["metrics"].data_ptr(), d_off.data_ptr(), None, out["valid"].data_ptr(),
                         d_seeds.data_ptr(), g[0].data_ptr(), g[1].data_ptr(), g[2].data_ptr())
    need = lib.pm_analyze_sweep_scratch_bytes(n, packed.max_phase_samples, G, 4, B)
    scratch = torch.empty(need, dtype=torch.uint8, device="cuda")
    rc = lib.pm_analyze_sweep_device(t, pol, res, job, C.c_void_p(scratch.data_ptr()), need - 1, None, None)
    assert rc == -1 and "scratch" in N.last_error()            # PM_E_INVALID
    rc = lib.pm_analyze_sweep_device(t, pol, res, job, C.c_void_p(scratch.data_ptr() + 8), need, None, None)
    assert rc == -1 and "aligned" in N.last_error()
