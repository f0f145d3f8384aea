"""Build libpmb200.so (every CUDA source under csrc/) for sm_100a, in tree.

``python -m powermodeling_b200.build`` compiles each translation unit with
nvcc into ``_build/`` and links ``powermodeling_b200/libpmb200.so``.  Sources
are recompiled only when they or a header changed.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libpmb200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: CPython rounds every multiply and add separately; the analysis
# kernels reproduce its arithmetic operation by operation.
COMMON = ["-std=c++17", "-O3", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC,-O2",
          "-I" + str(INCLUDE), "-I" + str(CSRC)]


# Compiled with contraction on, as the reference's nonlinear kernels are: the
# pointwise functions then round exactly as the reference's do.
FMAD_DEFAULT = {"nonlinear.cu"}


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libpmb200")
    return path


EXECUTABLE = PACKAGE / "bin" / "powerbench"
MAIN = CSRC / "powerbench_main.cpp"
# The record packer is a CPython extension (host C++, no CUDA).
PACKER_SRC = CSRC / "python" / "packer.cpp"
PACKER = PACKAGE / ("_packnative" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
# The record assembly helpers: a second CPython extension (host C++).
RECORDS_SRC = CSRC / "python" / "records.cpp"
RECORDS = PACKAGE / ("_recordnative" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(p for p in CSRC.glob("*.cpp") if p != MAIN)


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    objects, commands = [], []
    for src in _sources():
        obj = BUILD / (src.name + ".o")
        objects.append(obj)
        if _stale(obj, src, headers):
            extra = ARCH if src.suffix == ".cu" else []
            flags = [f for f in COMMON if f != "--fmad=false"] if src.name in FMAD_DEFAULT else COMMON
            commands.append([nvcc(), *flags, *extra, "-c", str(src), "-o", str(obj)])
    procs = []
    limit = jobs or max(1, min(8, os.cpu_count() or 1))
    for cmd in commands:
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
        if len(procs) >= limit:
            _drain(procs.pop(0))
    for p in procs:
        _drain(p)
    if commands or not LIBRARY.exists():
        link = [nvcc(), *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects),
                "-lcublas", "-lcuda", "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(link), file=sys.stderr)
        _drain(subprocess.Popen(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    if _stale(EXECUTABLE, MAIN, [LIBRARY, INCLUDE / "pmb200.h"]):
        EXECUTABLE.parent.mkdir(exist_ok=True)
        exe = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-I" + str(INCLUDE), str(MAIN), "-o", str(EXECUTABLE),
               "-L" + str(PACKAGE), "-lpmb200", "-Wl,-rpath,$ORIGIN/.."]
        if verbose:
            print(" ".join(exe), file=sys.stderr)
        _drain(subprocess.Popen(exe, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    for target, source in ((PACKER, PACKER_SRC), (RECORDS, RECORDS_SRC)):
        if _stale(target, source, [INCLUDE / "pmb200.h"]):
            ext = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-fvisibility=hidden",
                   "-I" + sysconfig.get_paths()["include"], "-I" + str(INCLUDE), str(source), "-o", str(target)]
            if verbose:
                print(" ".join(ext), file=sys.stderr)
            _drain(subprocess.Popen(ext, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    return LIBRARY


def _drain(proc: subprocess.Popen) -> None:
    out, _ = proc.communicate()
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed ({' '.join(proc.args[:2])} ...):\n{out}")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
