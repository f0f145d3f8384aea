"""The powerbench command line, in process or as the executable.

``run(args)`` calls libpmb200's pm_powerbench with the reference's powerbench
flags and returns the JSONL records it emitted; ``EXECUTABLE`` is the same
engine as a program for powermodeling's runner (``--bench``).
"""
from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

from . import _native as N

EXECUTABLE = Path(__file__).resolve().parent / "bin" / "powerbench"
_LINE = C.CFUNCTYPE(None, C.c_char_p, C.c_void_p)


class PowerbenchError(RuntimeError):
    """powerbench exited with status 1; ``records`` holds what it emitted first."""

    def __init__(self, message: str, records: list):
        super().__init__(message)
        self.records = records


def run(args: list[str]) -> list[dict]:
    lib = N.library()
    lib.pm_powerbench.argtypes = [C.c_int, C.POINTER(C.c_char_p), _LINE, C.c_void_p]
    lines: list[str] = []
    callback = _LINE(lambda line, _user: lines.append(line.decode()))
    argv = ["powerbench", *map(str, args)]
    arr = (C.c_char_p * len(argv))(*(a.encode() for a in argv))
    rc = lib.pm_powerbench(len(argv), arr, callback, None)
    records = [json.loads(line) for line in lines if not line.startswith("#")]
    if rc != 0:
        raise PowerbenchError(N.last_error(), records)
    return records


def tensor_probe(accumulators: int = 1, iterations: int = 1, uniform: bool = False, seed: int = 1):
    """Accumulator 0 of one tcgen05 CTA with its fp16 operands: (out [128,N], a [128,64], b [256,64])."""
    import numpy as np
    lib = N.library()
    lib.pm_tensor_probe.argtypes = [C.c_int, C.c_uint64, C.c_int, C.c_uint64, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
    n = min(256, (512 // accumulators) // 16 * 16)
    out = np.zeros((128, n), dtype=np.float32)
    a = np.zeros((128, 64), dtype=np.uint16)
    b = np.zeros((256, 64), dtype=np.uint16)
    N.check(lib.pm_tensor_probe(accumulators, iterations, int(uniform), seed, out.ctypes.data, out.size,
                                a.ctypes.data, b.ctypes.data), "pm_tensor_probe")
    return out, a.view(np.float16), b.view(np.float16)


def gemm_probe(m: int, n: int, k: int, uniform: bool = False, seed: int = 1):
    """The gemm arm's cuBLAS call once: (C [m, n], A [m, k], B [k, n]) as float32 / float16 arrays."""
    import numpy as np
    lib = N.library()
    lib.pm_gemm_probe.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p]
    out = np.zeros(m * n, dtype=np.float32)
    a = np.zeros(m * k, dtype=np.uint16)
    b = np.zeros(k * n, dtype=np.uint16)
    N.check(lib.pm_gemm_probe(m, n, k, int(uniform), seed, out.ctypes.data, a.ctypes.data, b.ctypes.data), "pm_gemm_probe")
    col = lambda x, rows, cols: x.reshape(cols, rows).T      # column-major storage
    return col(out, m, n), col(a.view(np.float16), m, k), col(b.view(np.float16), k, n)
