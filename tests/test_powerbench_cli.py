"""powerbench argv grammar: the reference's guards, checked before any CUDA call (CPU)."""
from __future__ import annotations

import subprocess

import pytest

from powermodeling_b200 import powerbench

REJECTED = [
    (["--workload", "hbm", "--threads", "33"], "--threads must be a multiple of 32"),
    (["--workload", "hbm", "--offset-bytes", "6"], "multiples of 4"),
    (["--workload", "hbm", "--stride-words", "1", "--stride-elements", "1"], "choose only one"),
    (["--workload", "hbm", "--stride-words", "0"], "invalid --stride-words"),
    (["--workload", "tensor", "--tensor-accumulators", "9"], "1..8"),
    (["--workload", "bogus"], "unknown workload"),
    (["--workload", "l1", "--access", "copy"], "L1 global-store/copy"),
    (["--workload", "l2_latency", "--stride-words", "2"], "randomized dependent links"),
    (["--workload", "gemm", "--sm-ids", "0,1"], "cannot honor --sm-ids"),
    (["--workload", "hbm", "--paired-reference", "--seconds", "2"], "paired energy arms require"),
    (["--workload", "sfu_ex2", "--grid-mode", "fixed"], "fixed nonlinear/SFU grid requires"),
    (["--workload", "sfu_ex2", "--sfu-chains", "3"], "--sfu-chains must be 1, 4 or 8"),
    (["--workload", "hbm", "--sfu-lanes", "64"], "apply only to register SFU"),
    (["--workload", "sfu_ex2", "--working-set-bytes", "4096"], "register SFU uses --sfu-lanes"),
    (["--workload", "control", "--grid-mode", "auto"], "applies only to nonlinear/SFU"),
    (["--workload", "hbm", "--reference-order", "CA"], "AB or BA"),
    (["--workload", "hbm", "--iterations", str(2 ** 32 + 1)], "<= 2^32"),
    (["--workload", "hbm", "--bogus", "1"], "unknown option"),
    (["--workload", "hbm", "--seconds"], "missing value"),
    (["--workload", "hbm", "--seconds", "-1"], "finite nonnegative"),
    (["--workload", "hbm", "--memory-vector-bytes", "8"], "must be 4 or 16"),
    (["--workload", "hbm", "--memory-vector-bytes", "16", "--offset-bytes", "4"], "multiple of 16"),
    # Complete streaming nonlinear functions (gpu_bench.cu:164-172, 226-247).
    (["--workload", "exp"], "require explicit --nonlinear-mode streaming"),
    (["--workload", "softmax", "--nonlinear-mode", "batched"], "require explicit --nonlinear-mode streaming"),
    (["--workload", "hbm", "--nonlinear-mode", "streaming"], "applies only to complete exp/tanh/silu/rmsnorm/softmax"),
    (["--workload", "exp", "--nonlinear-mode", "streaming", "--row-width", "16"], "--row-width 1..65536 applies only"),
    (["--workload", "rmsnorm", "--nonlinear-mode", "streaming", "--row-width", "65537"], "--row-width 1..65536 applies only"),
    (["--workload", "softmax", "--nonlinear-mode", "streaming", "--row-width", "0"], "--row-width must be positive"),
    (["--workload", "silu", "--nonlinear-mode", "streaming", "--access", "copy"], "require a full grid, offset=0"),
    (["--workload", "tanh", "--nonlinear-mode", "streaming", "--stride-words", "2"], "require a full grid, offset=0"),
    (["--workload", "exp", "--nonlinear-mode", "streaming", "--sm-ids", "0"], "require a full grid, offset=0"),
    (["--workload", "exp", "--nonlinear-mode", "streaming", "--grid-mode", "fixed"], "requires explicit positive --blocks"),
    (["--workload", "exp", "--nonlinear-mode", "streaming", "--grid-mode", "guess"], "--grid-mode must be auto or fixed"),
]
# The reference's cache-policy combinations (tests/test_memory_read_contract.py:272-285).
POLICY = [("hbm", "read", "bogus"), ("l1", "read", "cg"), ("l2", "read", "ca"), ("hbm", "write", "cg"),
          ("tensor", "read", "auto"), ("l2_latency", "read", "cg")]


@pytest.mark.parametrize("args,message", REJECTED)
def test_rejected_before_cuda(args, message):
    with pytest.raises(powerbench.PowerbenchError) as err:
        powerbench.run(args)
    assert message in str(err.value), str(err.value)
    assert "cuda" not in str(err.value).lower() or "CUDA" in message


@pytest.mark.parametrize("workload,access,policy", POLICY)
def test_cache_policy_combinations_fail_before_cuda(workload, access, policy):
    with pytest.raises(powerbench.PowerbenchError) as err:
        powerbench.run(["--workload", workload, "--access", access, "--read-cache-policy", policy])
    assert "read-cache-policy" in str(err.value)
    assert "unknown option" not in str(err.value)


def test_executable_reports_errors_on_stderr_with_status_1():
    proc = subprocess.run([str(powerbench.EXECUTABLE), "--workload", "hbm", "--threads", "7"], capture_output=True, text=True)
    assert proc.returncode == 1
    assert proc.stderr.startswith("powerbench: --threads must be a multiple of 32")
    assert proc.stdout == ""


def test_help_lists_the_reference_flags():
    proc = subprocess.run([str(powerbench.EXECUTABLE), "--help"], capture_output=True, text=True)
    assert proc.returncode == 0
    for flag in ("--working-set-bytes", "--stride-words", "--paired-reference", "--sfu-lanes", "--read-cache-policy",
                 "--nonlinear-mode", "--row-width"):
        assert flag in proc.stdout
