"""Build recipe for the checkers under oracle/ (test infrastructure only).

* ``oracle/liboracle_words.so`` from oracle/*.cpp: a CPU restatement of the
  reference's deterministic workload bookkeeping (word fill, read sums,
  checksums, pointer-chase permutation, SFU initial operands).
* ``oracle/_ref/powerbench_ref``: the reference's own powerbench compiled
  for sm_100a from its sources where they lie (cuda/gpu_bench.cu with its
  three headers) when the reference tree is present.  It is the bit-exact
  checker for values only the GPU can produce (MUFU approximations).  Nothing
  is copied from the reference tree; the binary is git-ignored.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _stale(target: Path, sources: list[Path]) -> bool:
    return not target.exists() or any(s.stat().st_mtime > target.stat().st_mtime for s in sources)


def build_words() -> Path | None:
    sources = sorted(HERE.glob("*.cpp"))
    if not sources:
        return None
    target = HERE / "liboracle_words.so"
    if _stale(target, sources):
        _run([shutil.which("g++") or "g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-o", str(target), *map(str, sources)])
    return target


def build_reference(tree: str | os.PathLike | None) -> Path | None:
    """``tree``: the reference checkout (None: nothing to build)."""
    if not tree:
        return None
    reference = Path(tree)
    source = reference / "cuda" / "gpu_bench.cu"
    if not source.exists():
        return None
    REF_OUT.mkdir(exist_ok=True)
    target = REF_OUT / "powerbench_ref"
    headers = [reference / "cuda" / h for h in ("sfu.cuh", "nonlinear.cuh", "memory_read_math.cuh")]
    if _stale(target, [source, *[h for h in headers if h.exists()]]):
        nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
        _run([nvcc, "-std=c++17", "-O3", "--expt-relaxed-constexpr", "-gencode", "arch=compute_100a,code=sm_100a",
              "-I", str(source.parent), str(source), "-o", str(target), "-lcublas"])
    return target


def build(tree: str | os.PathLike | None = None) -> None:
    """The word oracle always; the reference binary when ``tree`` (or PM_REFERENCE_TREE) names a checkout."""
    build_words()
    build_reference(tree or os.environ.get("PM_REFERENCE_TREE"))


if __name__ == "__main__":
    import sys
    build(sys.argv[1] if len(sys.argv) > 1 else None)
    print("oracle built")
