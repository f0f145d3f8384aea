"""Generate the golden telemetry fixtures from the reference implementation.

    python tests/golden/make_telemetry_golden.py <reference checkout>      (or PM_REFERENCE_TREE=<reference checkout>)

Runs the reference's NvmlDevice (powermodeling/telemetry.py) on every fake
driver scenario of tests/nvml_fake.py — read_sample repeated as the scenario
says, then capabilities and metadata() — and the reference's phase slicing
(powermodeling/runner.py _phase_records) on tests/nvml_fake.phase_cases().
Host timestamps are dropped; everything else is written to
tests/golden/telemetry.json.gz.
"""
from __future__ import annotations

import gzip
import json
import math
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import nvml_fake  # noqa: E402


def _clean(value):
    """JSON-safe copy: NaN becomes the string "nan"."""
    if isinstance(value, float) and math.isnan(value):
        return "nan"
    if isinstance(value, dict):
        return {k: _clean(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_clean(v) for v in value]
    return value


def sample_cases(NvmlDevice):
    out = {}
    for name, (factory, reads) in nvml_fake.SCENARIOS.items():
        fake = factory()
        case = {"reads": []}
        try:
            with NvmlDevice(nvml_module=fake) as device:
                for _ in range(reads):
                    case["reads"].append(nvml_fake.strip_timing(device.read_sample()))
                case["capabilities"] = json.loads(json.dumps(device.capabilities))
                meta = device.metadata()
                meta["sample"] = nvml_fake.strip_timing(meta["sample"])
                case["metadata"] = meta
        except Exception as exc:  # noqa: BLE001
            case["raises"] = [type(exc).__name__, str(exc)]
        out[name] = _clean(case)
    return out


def phase_outputs(phase_records):
    out = {}
    for name, (events, times) in nvml_fake.phase_cases().items():
        samples = [{"t_s": t, "i": i} for i, t in enumerate(times)]
        try:
            phases = phase_records(events, samples)
            out[name] = {"phases": {k: {"start_s": v["start_s"], "end_s": v["end_s"],
                                        "samples": [s["i"] for s in v["samples"]]} for k, v in phases.items()}}
        except Exception as exc:  # noqa: BLE001
            out[name] = {"raises": [type(exc).__name__, str(exc)]}
    return out


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from powermodeling.runner import _phase_records
    from powermodeling.telemetry import NvmlDevice
    data = {"samples": sample_cases(NvmlDevice), "phases": phase_outputs(_phase_records)}
    path = HERE / "telemetry.json.gz"
    with gzip.open(path, "wt") as f:
        json.dump(data, f, indent=0, sort_keys=True)
    print(path, len(data["samples"]), "scenarios", len(data["phases"]), "phase cases")


if __name__ == "__main__":
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PM_REFERENCE_TREE")
    if not tree:
        sys.exit(f"usage: {Path(__file__).name} <reference checkout>  (or set PM_REFERENCE_TREE)")
    main(tree)
