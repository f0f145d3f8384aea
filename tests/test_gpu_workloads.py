"""GPU parity of the workload arms: checksums against the oracle and the reference's powerbench."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

import workload_oracle as W
from powermodeling_b200 import contracts, powerbench
from test_oracle_words import READ_CASES, reference_digest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
REF_BIN = ROOT / "oracle" / "_ref" / "powerbench_ref"
QUICK = ["--seconds", "0.05", "--warmup-seconds", "0", "--idle-seconds", "0", "--batch-launches", "1", "--fixed-batches", "2"]


def result_of(records, kind="result"):
    found = [r for r in records if r.get("type") == kind]
    assert len(found) == 1, [r.get("type") for r in records]
    return found[0]


def reference_result(args, required: bool = False):
    """The reference's own powerbench (built from its sources for sm_100a) on the same arguments.

    required: the reference binary is the only checker (SFU checksums depend on
    the hardware's MUFU approximations), so its absence fails the test."""
    if not REF_BIN.exists():
        if required:
            pytest.fail(f"{REF_BIN.relative_to(ROOT)} is missing: build it with oracle/build_oracle.py")
        return None
    proc = subprocess.run([str(REF_BIN), *map(str, args)], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr
    return result_of([json.loads(line) for line in proc.stdout.splitlines()])


def test_describe_record(gpu_ready):
    dev = result_of(powerbench.run(["--describe"]), "device")
    assert dev["uuid"].startswith("GPU-") and dev["compute_capability_major"] == 10
    assert dev["sm_count"] >= 1 and dev["memory_bus_width_bits"] > 0


@pytest.mark.parametrize("workload,words,iterations,stride,offset", READ_CASES)
def test_scalar_read_sums_match_reference_cases(gpu_ready, workload, words, iterations, stride, offset):
    args = ["--workload", workload, "--access", "read", "--blocks", "2", "--threads", "32",
            "--working-set-bytes", words * 4, "--stride-elements", stride, "--offset-bytes", offset, "--seed", "7",
            "--iterations", iterations, *QUICK]
    r = result_of(powerbench.run(args))
    assert r["kernel_implementation_version"] == "scalar_single_stream_read_v3"
    assert r["memory_read_index_math"] == "uint32"
    assert r["read_cache_policy"] == ("ca" if workload == "l1" else "cg")
    assert r["admitted_blocks"] == 4 and r["operations"] == 4 * 32 * iterations
    assert sum(e["operations"] for e in r["measure_epochs"]) == r["operations"]
    assert r["checksum"] == reference_digest(workload, words, iterations, stride, offset)
    assert r["memory_read_validation"]["status"] == "pass" and r["memory_read_validation"]["mismatched_values"] == 0
    assert contracts.memory_count_issues(r, workload) == []
    ref = reference_result(args)
    if ref is not None:
        assert ref["checksum"] == r["checksum"]


@pytest.mark.parametrize("policy", ["cg", "cs", "ca"])
def test_hbm_scalar_and_vector_reads(gpu_ready, policy):
    base = ["--workload", "hbm", "--blocks", "8", "--threads", "64", "--working-set-bytes", 1 << 20, "--seed", "11",
            "--iterations", "33", "--stride-words", "3", "--offset-bytes", "32", "--read-cache-policy", policy, *QUICK]
    scalar = result_of(powerbench.run(base))
    words = (1 << 20) // 4
    sums = W.read_sums(words, 8, 11, 8, 64, 3, 33)
    assert scalar["checksum"] == W.sink_hash(sums[:512])
    vector = result_of(powerbench.run(base + ["--memory-vector-bytes", "16"]))
    assert vector["kernel_implementation_version"] == "vector_quad_single_stream_read_v1"
    assert vector["logical_bytes"] == vector["operations"] * 16
    vsums = W.read_sums(words, 8, 11, 8, 64, 3, 33, unit=4)
    assert vector["checksum"] == W.sink_hash(vsums[:512])
    assert vector["memory_read_validation"]["status"] == "pass"
    ref = reference_result(base)
    if ref is not None:
        assert ref["checksum"] == scalar["checksum"]


@pytest.mark.parametrize("vector", [False, True])
def test_lcg_fill_read_sums(gpu_ready, vector):
    """The seeded uint32 LCG payload (an extra mode): per-thread read sums equal the oracle's over
    the stepped recurrence, and the engine's own CPU check passes."""
    words, blocks, threads, stride, iters = (1 << 20) // 4, 8, 64, 3, 33
    args = ["--workload", "hbm", "--fill", "lcg", "--blocks", blocks, "--threads", threads, "--working-set-bytes", 1 << 20,
            "--seed", "11", "--iterations", iters, "--stride-words", stride, "--offset-bytes", "32", *QUICK]
    r = result_of(powerbench.run(args + (["--memory-vector-bytes", "16"] if vector else [])))
    assert r["memory_fill"] == "uint32_lcg_1664525_1013904223_v1"
    assert r["memory_read_validation"]["status"] == "pass"
    sums = W.read_sums_of(W.lcg_words(words + 8, 11), words, 8, blocks, threads, stride, iters, unit=4 if vector else 1)
    assert r["checksum"] == W.sink_hash(sums[:512])
    plain = result_of(powerbench.run(args[:2] + args[4:]))
    assert plain["memory_fill"] == "random_word_xor_seed_v1" and plain["checksum"] != r["checksum"]


@pytest.mark.parametrize("workload", ["sfu_ex2", "sfu_rsqrt", "sfu_tanh"])
def test_sfu_uniform_input_mode(gpu_ready, workload):
    """Operands uniform in [0.5, 2) with a per-thread XOR checksum (an extra mode): the one-step
    checks pass on the new operands, the XOR fold is deterministic, and the record names the mode."""
    args = ["--workload", workload, "--threads", "256", "--sfu-lanes", "8192", "--sfu-chains", "4", "--iterations", "64",
            "--seed", "5", "--sfu-input", "uniform_0p5_2", *QUICK]
    r = result_of(powerbench.run(args))
    assert r["sanity"]["numerical_validation_passed"] is True and r["numerical_validation"]["checked_values"] == 16
    assert r["sfu_input_policy"] == "thread_hash_uniform_0p5_2_then_feedback_xor_iteration_mantissa_0p5_1_v1"
    assert r["checksum_kind"] == "distributed_per_lane_register_xor_sample"
    again = result_of(powerbench.run(args))
    assert isinstance(r["sfu_thread_xor_checksum"], int) and r["sfu_thread_xor_checksum"] == again["sfu_thread_xor_checksum"]
    assert again["checksum"] == r["checksum"]
    parity = result_of(powerbench.run([a for a in args if a not in ("--sfu-input", "uniform_0p5_2")]))
    assert parity["sfu_thread_xor_checksum"] is None and parity["checksum"] != r["checksum"]


@pytest.mark.parametrize("access,vector", [("copy", False), ("write", False), ("copy", True)])
def test_write_copy_sinks(gpu_ready, access, vector):
    blocks, threads, stride, iters = 4, 64, 3, 7
    args = ["--workload", "hbm", "--access", access, "--blocks", blocks, "--threads", threads,
            "--working-set-bytes", 1 << 20, "--stride-words", stride, "--offset-bytes", "16", "--seed", "5",
            "--iterations", iters, *QUICK] + (["--memory-vector-bytes", "16"] if vector else [])
    r = result_of(powerbench.run(args))
    lanes = blocks * threads
    if vector:
        quads = r["working_set_bytes"] // 16
        sinks = W.copy_vector_sinks(quads, 4, 5, blocks, threads, stride, iters)
        assert r["logical_bytes"] == r["operations"] * 32
    else:
        sinks = W.write_copy_sinks(r["working_set_bytes"] // 4, 4, 5, blocks, threads, stride, iters, access == "copy")
        assert contracts.memory_count_issues(r, "hbm") == []
        ref = reference_result(args)
        if ref is not None:
            assert ref["checksum"] == r["checksum"]
    assert r["checksum"] == W.sink_hash(sinks[:min(1024, lanes)])


def test_control_issue_loop(gpu_ready):
    args = ["--workload", "control", "--blocks", "3", "--threads", "96", "--iterations", "1000", *QUICK]
    r = result_of(powerbench.run(args))
    assert r["checksum"] == W.sink_hash(W.control_sinks(1000, 288))
    ref = reference_result(args)
    if ref is not None:
        assert ref["checksum"] == r["checksum"]


def test_word_chase_terminals(gpu_ready):
    blocks, threads, nodes, iters, seed = 5, 32, 100003, 1000, 9
    args = ["--workload", "l2_latency", "--blocks", blocks, "--threads", threads, "--working-set-bytes", nodes * 4,
            "--iterations", iters, "--seed", seed, *QUICK]
    r = result_of(powerbench.run(args))
    links = W.chase_links(nodes, seed)
    sink = np.zeros(blocks * threads, dtype=np.uint32)
    for b in range(blocks):
        sink[b * threads] = W.chase_terminal(links, iters, seed + 2, b)   # last measured launch: nonce seed + 2
    assert r["checksum"] == W.sink_hash(sink)
    probe = r["latency_probe"]["per_sm"]
    assert probe and all(v["cycles_per_access"] > 0 for v in probe.values())
    ref = reference_result(args)
    if ref is not None:
        assert ref["checksum"] == r["checksum"]


def test_line_chase_terminals(gpu_ready):
    blocks, nodes, iters, seed = 148, 4096, 2000, 21
    args = ["--workload", "l2_latency", "--chase-granularity", "line", "--blocks", blocks, "--threads", "32",
            "--working-set-bytes", nodes * 128, "--iterations", iters, "--seed", seed, *QUICK]
    r = result_of(powerbench.run(args))
    links = W.chase_links(nodes, seed)
    term = np.array([W.chase_terminal(links, iters, seed + 2, b) for b in range(blocks)], dtype=np.uint64)
    assert r["checksum"] == int(W.lib().oracle_u64_hash(term.ctypes.data, term.size))
    assert r["logical_bytes"] == r["operations"] * 8


@pytest.mark.parametrize("workload", ["sfu_ex2", "sfu_lg2", "sfu_rcp", "sfu_rsqrt", "sfu_sqrt", "sfu_tanh"])
def test_sfu_arms(gpu_ready, workload):
    args = ["--workload", workload, "--threads", "256", "--sfu-lanes", "8192", "--sfu-chains", "4", "--iterations", "256",
            "--seed", "3", *QUICK]
    r = result_of(powerbench.run(args))
    assert r["numerical_validation"]["checked_values"] == 16 and r["sanity"]["numerical_validation_passed"] is True
    assert contracts.sfu_count_issues(r, workload) == []
    assert r["kernel_resources"]["local_bytes_per_thread"] == 0
    ref = reference_result(args, required=True)
    assert ref["checksum"] == r["checksum"], workload


@pytest.mark.parametrize("accumulators,iterations,uniform", [(1, 1, False), (3, 2, True), (8, 5, True), (2, 1, True)])
def test_tcgen05_probe_matches_fp32_product(gpu_ready, accumulators, iterations, uniform):
    out, a, b = powerbench.tensor_probe(accumulators, iterations, uniform, seed=17)
    n = out.shape[1]
    ref = (a.astype(np.float64) @ b.astype(np.float64)[:n].T) * iterations
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64)[:n]).T * iterations
    assert np.all(np.abs(out - ref) <= 1e-5 * scale + 1e-6), float(np.max(np.abs(out - ref)))


def test_tensor_workload_counts(gpu_ready):
    args = ["--workload", "tensor", "--blocks", "148", "--threads", "128", "--iterations", "64",
            "--tensor-accumulators", "4", *QUICK]
    r = result_of(powerbench.run(args))
    assert r["tensor_status"]["bounded_wait_timeouts"] == 0
    assert r["sanity"]["finite_output_sample"] is True
    assert r["operations"] == r["admitted_blocks"] * 64 * 4 * 4 * 2 * 128 * 128 * 16


def test_gemm_arm_runs(gpu_ready):
    r = result_of(powerbench.run(["--workload", "gemm", "--gemm-m", "512", "--gemm-n", "512", "--gemm-k", "512", *QUICK]))
    assert r["operations"] == 2 * 2 * 512 ** 3 and r["sanity"]["finite_output_sample"] is True


@pytest.mark.parametrize("m,n,k,uniform", [(512, 512, 512, False), (256, 384, 1024, True), (512, 64, 4096, True)])
def test_gemm_arm_matches_fp64_product(gpu_ready, m, n, k, uniform):
    """cuBLAS fp16 x fp16 -> fp32 against the fp64 product of the same operands.

    fp16 products are exact in fp32, so the error is the fp32 accumulation's:
    within 1e-5 of sum |a||b| (the tcgen05 probe's tolerance)."""
    c, a, b = powerbench.gemm_probe(m, n, k, uniform, seed=23)
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    ref = a64 @ b64
    scale = np.abs(a64) @ np.abs(b64)
    assert np.all(np.isfinite(c))
    assert np.all(np.abs(c - ref) <= 1e-5 * scale + 1e-6), float(np.max(np.abs(c - ref) / (scale + 1e-30)))
