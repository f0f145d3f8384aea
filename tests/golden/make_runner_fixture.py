"""Records of this engine checked by the reference's own runner and count contracts.

Three steps, each writing a committed fixture:

    python tests/golden/make_runner_fixture.py plan <reference checkout>
        The reference's planner.benchmark_command (planner.py:660-682) turns
        the trials below into powerbench argv lists -> tests/golden/runner_plan.json
    python tests/golden/make_runner_fixture.py capture OUT.json.gz      (on a B200)
        Runs every argv through this package's powerbench under its native
        NVML sampler (capture.capture_trial, 50 ms, the reference's default
        interval) and keeps the raw stdout lines, samples, device metadata and
        pid -> tests/golden/runner_captures.json.gz
    python tests/golden/make_runner_fixture.py check <reference checkout>
        Replays each capture through the reference's runner.capture_trial
        (runner.py:331-480: one result, protocol and device per trial, UUID
        match, ordered phases, paired-protocol checks, exclusivity) with its
        subprocess and sampler replaced by the stored stdout and samples, and
        runs sfu/memory/nonlinear.count_issues -> tests/golden/runner_checks.json.gz;
        keeps the runner's records with the reference's analyze_trial of each
        and its summarize over all of them -> tests/golden/runner_records.json.gz

PM_REFERENCE_TREE may name the reference checkout instead of the argument.
"""
from __future__ import annotations

import gzip
import json
import os
import subprocess
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

# (trial_id, workload, parameters, paired order or None): short arms of every workload family.
TRIALS = [
    ("hbm-read-scalar", "hbm", {"blocks": 296, "threads": 256, "working_set_bytes": 1 << 30, "iterations": 512}, None),
    ("hbm-read-vector", "hbm", {"blocks": 1184, "threads": 256, "working_set_bytes": 1 << 30, "iterations": 128,
                                "memory_vector_bytes": 16, "read_cache_policy": "cs"}, None),
    ("hbm-copy", "hbm", {"access": "copy", "blocks": 592, "threads": 256, "working_set_bytes": 1 << 30,
                         "iterations": 64}, None),
    ("l2-read", "l2", {"blocks": 296, "threads": 256, "working_set_bytes": 32 << 20, "iterations": 1024}, None),
    ("l1-read", "l1", {"blocks": 148, "threads": 256, "working_set_bytes": 148 * 65536, "iterations": 2048}, None),
    ("chase-words", "l2_latency", {"blocks": 148, "threads": 32, "working_set_bytes": 16 << 20, "iterations": 20000}, None),
    ("tensor", "tensor", {"blocks": 148, "threads": 128, "iterations": 2048, "tensor_accumulators": 2}, None),
    ("gemm", "gemm", {"gemm_m": 2048, "gemm_n": 2048, "gemm_k": 2048}, None),
    ("control", "control", {"blocks": 296, "threads": 256, "iterations": 4096}, None),
    ("sfu-ex2-paired", "sfu_ex2", {"grid_mode": "fixed", "blocks": 1184, "threads": 256, "sfu_lanes": 1184 * 256,
                                   "sfu_chains": 4, "iterations": 4096}, "AB"),
    ("sfu-tanh", "sfu_tanh", {"sfu_lanes": 65536, "threads": 256, "sfu_chains": 8, "iterations": 4096}, None),
    ("softmax-paired", "softmax", {"nonlinear_mode": "streaming", "row_width": 1024, "grid_mode": "fixed",
                                   "blocks": 1184, "threads": 256, "working_set_bytes": 1 << 28}, "BA"),
    ("rmsnorm", "rmsnorm", {"nonlinear_mode": "streaming", "row_width": 1024, "working_set_bytes": 1 << 28}, None),
    ("exp", "exp", {"nonlinear_mode": "streaming", "working_set_bytes": 1 << 28}, None),
]
SECONDS, WARMUP, IDLE, INTERVAL = 1.0, 0.2, 0.5, 0.05
# Paired trials run the reference's minimum arms (the engine refuses shorter ones, gpu_bench.cu's guard).
PAIRED_SECONDS, PAIRED_WARMUP, PAIRED_IDLE = 10.0, 1.0, 6.0


def plan_trials() -> list[dict]:
    out = []
    for trial_id, workload, parameters, order in TRIALS:
        trial = {"trial_id": trial_id, "condition_id": trial_id, "repeat": 0, "workload": workload,
                 "experiment_role": "energy_candidate", "parameters": dict(parameters),
                 "clocks": {"graphics_mhz": None, "memory_mhz": None}, "seconds": SECONDS,
                 "warmup_seconds": WARMUP, "idle_seconds": IDLE, "stage": "runner_contract_fixture"}
        if order:
            trial["treatment_protocol"] = {"kind": "paired_active_reference", "order": order}
            trial.update(seconds=PAIRED_SECONDS, warmup_seconds=PAIRED_WARMUP, idle_seconds=PAIRED_IDLE)
        out.append(trial)
    return out


def _reference(tree: str | None) -> str:
    tree = tree or os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit("name the reference checkout (argument or PM_REFERENCE_TREE)")
    sys.path.insert(0, tree)
    return tree


def make_plan(tree: str | None) -> None:
    _reference(tree)
    from powermodeling.planner import benchmark_command
    plan = [{"trial": t, "argv": benchmark_command("powerbench", t, 0)[1:]} for t in plan_trials()]
    (HERE / "runner_plan.json").write_text(json.dumps(plan, indent=1) + "\n")
    print(f"{len(plan)} trials planned")


def capture(out_path: str) -> None:
    """On a B200: every planned argv through this engine, captured under the native sampler."""
    sys.path.insert(0, str(ROOT))
    from powermodeling_b200 import powerbench
    from powermodeling_b200.capture import capture_trial
    from powermodeling_b200.telemetry import NvmlDevice
    plan = json.loads((HERE / "runner_plan.json").read_text())
    cuda = next(r for r in powerbench.run(["--describe"]) if r["type"] == "device")
    device = NvmlDevice(uuid=cuda["uuid"])
    out = []
    try:
        for entry in plan:
            record = capture_trial(entry["argv"], device, sample_interval_s=INTERVAL, trial_id=entry["trial"]["trial_id"])
            out.append({"trial_id": entry["trial"]["trial_id"],
                        "stdout": "".join(json.dumps(e) + "\n" for e in record["events"]),
                        "exit_code": record["quality"]["benchmark_exit_code"],
                        "pid": record["quality"]["measurement_pid"], "samples": record["samples"],
                        "device_metadata": record["device"], "uuid": cuda["uuid"],
                        "own_runner_errors": record["quality"]["runner_errors"]})
            print(entry["trial"]["trial_id"], record["status"], record["quality"]["runner_errors"], flush=True)
    finally:
        device.close()
    with gzip.open(out_path, "wt") as f:
        json.dump(out, f)


class _Replay:
    """Stands in for subprocess.Popen: the stored stdout, exit code and pid of one capture."""

    def __init__(self, capture):
        self.capture, self.pid, self.returncode = capture, capture["pid"], None

    def communicate(self, timeout=None):
        self.returncode = self.capture["exit_code"]
        return self.capture["stdout"], ""

    def poll(self):
        return self.returncode


def check(tree: str | None) -> None:
    """The reference's runner and count contracts over the stored captures."""
    _reference(tree)
    import powermodeling.runner as runner
    import powermodeling.telemetry as telemetry
    from powermodeling import analysis, memory, nonlinear, sfu
    plan = {e["trial"]["trial_id"]: e["trial"] for e in json.loads((HERE / "runner_plan.json").read_text())}
    with gzip.open(HERE / "runner_captures.json.gz", "rt") as f:
        captures = json.load(f)
    results, records = [], []
    for cap in captures:
        class Sampler:
            def __init__(self, device, interval_s=0.05):
                self.samples = []

            def start(self):
                return self

            def stop(self, _samples=cap["samples"]):
                return list(_samples)

        class Device:
            uuid = cap["uuid"]

            def metadata(self, _meta=cap["device_metadata"]):
                return dict(_meta)

        # The runner's own module of subprocess calls, with Popen replaying this capture.
        runner.subprocess = types.SimpleNamespace(Popen=lambda *a, _cap=cap, **k: _Replay(_cap), PIPE=subprocess.PIPE,
                                                  TimeoutExpired=subprocess.TimeoutExpired, run=subprocess.run)
        telemetry.Sampler = Sampler
        record = runner.capture_trial("powerbench", plan[cap["trial_id"]], Device(),
                                      {"uuid": cap["uuid"], "device_index": 0}, sample_interval_s=INTERVAL)
        workload = plan[cap["trial_id"]]["workload"]
        bench, reference = record.get("benchmark") or {}, record.get("active_reference") or {}
        results.append({"trial_id": cap["trial_id"], "status": record["status"],
                        "runner_errors": record["quality"]["runner_errors"],
                        "exclusivity_verified": record["quality"].get("exclusivity_verified"),
                        "phases": sorted(record.get("phases", {})),
                        "sfu": sfu.count_issues(bench, workload),
                        "sfu_reference": sfu.count_issues(reference, workload, reference=True) if reference else [],
                        "memory": memory.count_issues(bench, workload),
                        "nonlinear": nonlinear.count_issues(bench, workload)})
        records.append(json.loads(json.dumps(record)))
        print(cap["trial_id"], record["status"], record["quality"]["runner_errors"])
    with gzip.open(HERE / "runner_checks.json.gz", "wt") as f:
        json.dump(results, f, indent=0, sort_keys=True)
    # JSON round trips: NaN and infinities travel as the json module writes them.
    analysed = [json.loads(json.dumps(analysis.analyze_trial(r))) for r in records]
    summary = json.loads(json.dumps(analysis.summarize(records)))
    with gzip.open(HERE / "runner_records.json.gz", "wt") as f:
        json.dump({"records": records, "trials": analysed, "groups": summary["groups"]}, f)
    print(sum(t["valid"] for t in analysed), "of", len(analysed), "trials valid;", len(summary["groups"]), "groups")


if __name__ == "__main__":
    step = sys.argv[1] if len(sys.argv) > 1 else ""
    arg = sys.argv[2] if len(sys.argv) > 2 else None
    if step == "plan":
        make_plan(arg)
    elif step == "capture":
        capture(arg or "runner_captures.json.gz")
    elif step == "check":
        check(arg)
    else:
        sys.exit(__doc__)
