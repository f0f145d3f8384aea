"""bench.py --impl reference: the reference arm's JSON line (CPU, no GPU needed)."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                          capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)


def test_rank_zero_prints_one_contract_line():
    proc = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "bootstrap resamples/s" and d["unit"] == "resamples/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "resamples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_other_ranks_exit_without_work():
    proc = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert not [l for l in proc.stdout.splitlines() if l.startswith("{")]
