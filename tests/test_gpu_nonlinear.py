"""GPU parity of the streaming nonlinear workloads (exp, tanh, silu, softmax, RMSNorm).

Through the C-ABI (pm_nonlinear_fill_device / pm_nonlinear_apply_device):
the device fill equals the oracle's bit for bit, and every output element is
within the reference's tolerance of the oracle's double result
(|y - e| <= 2e-6 + 2e-4 |e|, softmax rows summing to 1 within 2e-4) over
pointwise tails, row widths on both sides of the shared-memory staging
limit, auto and fixed grids, and 32..1024 threads.  Through powerbench: the
records pass the nonlinear count contract, and the pointwise checksums equal
those of the reference's own powerbench on the same arguments.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import nonlinear_oracle as O
from powermodeling_b200 import contracts, powerbench
from test_gpu_workloads import QUICK, reference_result, result_of

pytestmark = pytest.mark.gpu
FN = {"exp": 0, "tanh": 1, "silu": 2, "softmax": 3, "rmsnorm": 4}


def device_apply(function, n, seed, *, width=0, blocks=None, threads=256, iterations=1):
    import torch
    from powermodeling_b200 import _native as N
    lib = N.library()
    x = torch.empty(max(n, 4), dtype=torch.float32, device="cuda")
    g = torch.empty(max(width, 4), dtype=torch.float32, device="cuda")
    y = torch.full((max(n, 4),), float("nan"), dtype=torch.float32, device="cuda")
    N.check(lib.pm_nonlinear_fill_device(C.c_void_p(x.data_ptr()), n, seed, 100.0 if function == "softmax" else 0.0, 0, None), "fill")
    N.check(lib.pm_nonlinear_fill_device(C.c_void_p(g.data_ptr()), max(width, 1), seed ^ 12345, 0.0, 1, None), "fill")
    if blocks is None:
        blocks = n // width if width else -(-n // threads)
    N.check(lib.pm_nonlinear_apply_device(FN[function], C.c_void_p(x.data_ptr()), C.c_void_p(g.data_ptr()),
                                          C.c_void_p(y.data_ptr()), n, width, iterations, blocks, threads, None), "apply")
    torch.cuda.synchronize()
    return x[:n].cpu().numpy(), g[:max(width, 1)].cpu().numpy(), y[:n].cpu().numpy()


@pytest.mark.parametrize("seed", [1, 7, 2 ** 40 + 3])
def test_device_fill_equals_oracle(gpu_ready, seed):
    import torch
    from powermodeling_b200 import _native as N
    lib = N.library()
    buf = torch.empty(3001, dtype=torch.float32, device="cuda")
    for shift, gamma in ((0.0, 0), (100.0, 0), (0.0, 1)):
        N.check(lib.pm_nonlinear_fill_device(C.c_void_p(buf.data_ptr()), 3001, seed, shift, gamma, None), "fill")
        got = buf.cpu().numpy()
        want = O.fill(3001, seed, shift, gamma=bool(gamma))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (shift, gamma)


POINTWISE = [(f, n, t, b) for f in ("exp", "tanh", "silu")
             for n, t, b in ((1, 96, None), (95, 96, None), (97, 96, None), (205, 96, None), (4099, 256, None),
                             (97, 96, 1), (97, 96, 3), (1 << 20, 256, 148), (1 << 20, 1024, 296), (12345, 32, 8))]


@pytest.mark.parametrize("function,n,threads,blocks", POINTWISE)
def test_pointwise_within_reference_tolerance(gpu_ready, function, n, threads, blocks):
    x, _, y = device_apply(function, n, 11, threads=threads, blocks=blocks)
    ok = O.within_tolerance(y, O.expected(function, x))
    assert ok.all(), (function, np.flatnonzero(~ok)[:5])


ROWWISE = [(f, w, rows, t, b) for f in ("softmax", "rmsnorm")
           for w, rows, t, b in ((1, 5, 96, None), (3, 7, 32, None), (129, 3, 96, None), (129, 5, 96, 2),
                                 (1024, 5, 96, None), (1024, 300, 256, 148), (4096, 37, 1024, None),
                                 (40960, 3, 256, None), (40961, 2, 96, None), (65536, 2, 512, 1), (5000, 9, 64, 4),
                                 # one CTA per row, row in registers: 1, 2 and 4 quads per thread
                                 (128, 9, 32, None), (2048, 5, 256, None), (1024, 6, 96, None), (16384, 2, 1024, None),
                                 # one warp per row: fixed grids with at least one row per warp
                                 (4, 1000, 64, 3), (128, 700, 96, 5), (256, 999, 256, 2), (512, 613, 1024, 1),
                                 (516, 300, 128, 2), (1024, 2000, 256, 7), (1024, 2000, 1024, 1), (1020, 97, 32, 3))]


@pytest.mark.parametrize("function,width,rows,threads,blocks", ROWWISE)
def test_rowwise_within_reference_tolerance(gpu_ready, function, width, rows, threads, blocks):
    x, g, y = device_apply(function, width * rows, 5, width=width, threads=threads, blocks=blocks)
    e = O.expected(function, x, g, width)
    ok = O.within_tolerance(y, e)
    assert ok.all(), (function, width, np.flatnonzero(~ok)[:5])
    if function == "softmax":
        assert O.softmax_rows_sum_to_one(y, width).all()


@pytest.mark.parametrize("function,width", [("exp", 0), ("silu", 0), ("softmax", 1024), ("rmsnorm", 129)])
def test_repeated_applications_rewrite_the_same_outputs(gpu_ready, function, width):
    n = 129 * 40 if width == 129 else 1024 * 33
    _, _, once = device_apply(function, n, 9, width=width, blocks=7)
    _, _, thrice = device_apply(function, n, 9, width=width, blocks=7, iterations=3)
    assert np.array_equal(once.view(np.uint32), thrice.view(np.uint32))


def test_large_softmax_rows_sum_to_one(gpu_ready):
    """A 1 GiB input (2^18 rows of 1024): every row sums to 1; sampled rows match the oracle."""
    import torch
    from powermodeling_b200 import _native as N
    lib = N.library()
    width, rows = 1024, 1 << 18
    n = width * rows
    x = torch.empty(n, dtype=torch.float32, device="cuda")
    y = torch.empty(n, dtype=torch.float32, device="cuda")
    N.check(lib.pm_nonlinear_fill_device(C.c_void_p(x.data_ptr()), n, 4, 100.0, 0, None), "fill")
    N.check(lib.pm_nonlinear_apply_device(3, C.c_void_p(x.data_ptr()), None, C.c_void_p(y.data_ptr()), n, width, 1,
                                          148 * 8, 256, None), "apply")
    sums = y.view(rows, width).double().sum(dim=1)
    assert float((sums - 1).abs().max()) <= 2e-4
    for r in O.sample_items(rows):
        xs = x[r * width:(r + 1) * width].cpu().numpy()
        assert O.within_tolerance(y[r * width:(r + 1) * width].cpu().numpy(), O.expected("softmax", xs, None, width)).all()
    del x, y
    torch.cuda.empty_cache()


def test_bad_arguments_are_rejected(gpu_ready):
    from powermodeling_b200 import _native as N
    lib = N.library()
    import torch
    buf = torch.empty(64, dtype=torch.float32, device="cuda")
    p = C.c_void_p(buf.data_ptr())
    odd = C.c_void_p(buf.data_ptr() + 4)
    assert lib.pm_nonlinear_apply_device(7, p, p, p, 16, 0, 1, 1, 32, None) == -1
    assert lib.pm_nonlinear_apply_device(0, odd, p, p, 16, 0, 1, 1, 32, None) == -1
    assert lib.pm_nonlinear_apply_device(3, p, p, p, 16, 5, 1, 1, 32, None) == -1      # partial row
    assert lib.pm_nonlinear_apply_device(0, p, p, p, 16, 4, 1, 1, 32, None) == -1      # width on a pointwise function
    assert lib.pm_nonlinear_apply_device(4, p, None, p, 16, 4, 1, 1, 32, None) == -1   # RMSNorm without gamma
    assert lib.pm_nonlinear_apply_device(0, p, p, p, 16, 0, 1, 1, 48, None) == -1      # threads not a multiple of 32


def run_arm(workload, elements, *, threads=96, width=129, grid_mode="auto", blocks=None, seed=1):
    args = ["--workload", workload, "--nonlinear-mode", "streaming", "--grid-mode", grid_mode, "--threads", threads,
            "--iterations", 2, "--working-set-bytes", elements * 4, "--seed", seed, *QUICK]
    if blocks is not None:
        args += ["--blocks", blocks]
    if workload in O.ROW_FUNCTIONS:
        args += ["--row-width", width]
    r = result_of(powerbench.run(args))
    assert contracts.nonlinear_count_issues(r, workload) == []
    assert r["elements"] == 4 * elements and r["input_elements"] == elements
    assert r["kernel_implementation_version"] == "fp32_complete_nonlinear_q_grid_v2"
    assert r["block_completion_count_source"] == "synchronized_completed_launches"
    assert r["admitted_blocks"] == 2 * r["blocks"]
    assert r["numerical_validation"]["checked_values"] > 0
    assert r["sanity"]["numerical_validation_passed"] is True and r["sanity"]["finite_output_sample"] is True
    assert r["kernel_resources"]["local_bytes_per_thread"] == 0
    return r, args


@pytest.mark.parametrize("workload", ["exp", "tanh", "silu"])
def test_pointwise_arm_tails_and_grids(gpu_ready, workload):
    for elements in (1, 95, 96, 97, 205):
        r, args = run_arm(workload, elements)
        assert r["blocks"] == (elements + 95) // 96
        ref = reference_result(args)
        if ref is not None:
            assert ref["checksum"] == r["checksum"], (workload, elements)
    for blocks in (1, 3, 8):
        r, args = run_arm(workload, 97, grid_mode="fixed", blocks=blocks)
        ref = reference_result(args)
        if ref is not None:
            assert ref["checksum"] == r["checksum"], (workload, blocks)


@pytest.mark.parametrize("workload", ["softmax", "rmsnorm"])
def test_rowwise_arm_rows_and_grids(gpu_ready, workload):
    for width in (1, 129, 1024):
        for rows in (1, 3, 5):
            r, args = run_arm(workload, rows * width, width=width)
            assert r["blocks"] == rows and r["row_evaluations"] == 4 * rows
            ref = reference_result(args)
            if ref is not None:
                assert ref["sanity"]["numerical_validation_passed"] is True
                assert ref["numerical_validation"]["checked_values"] == r["numerical_validation"]["checked_values"]
            run_arm(workload, rows * width, width=width, grid_mode="fixed", blocks=2)


@pytest.mark.parametrize("workload,extra,reason", [
    ("exp", ["--threads", "96", "--working-set-bytes", "388", "--blocks", "3"], "Q-derived auto grid"),
    ("softmax", ["--row-width", "129", "--working-set-bytes", "520"], "complete rows"),
])
def test_arm_rejects_conflicting_grids_and_partial_rows(gpu_ready, workload, extra, reason):
    with pytest.raises(powerbench.PowerbenchError) as err:
        powerbench.run(["--workload", workload, "--nonlinear-mode", "streaming", *extra])
    assert reason in str(err.value)
