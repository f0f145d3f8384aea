"""ctypes access to the C workload oracle (oracle/liboracle_words.so) for the tests."""
from __future__ import annotations

import ctypes as C
from functools import lru_cache
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent


@lru_cache(maxsize=1)
def lib():
    import oracle.build_oracle as ob
    path = ob.build_words()
    L = C.CDLL(str(path))
    u64, p = C.c_uint64, C.c_void_p
    L.oracle_random_word.restype = C.c_uint32
    L.oracle_random_word.argtypes = [u64]
    L.oracle_sink_hash.restype = u64
    L.oracle_sink_hash.argtypes = [p, u64]
    L.oracle_u64_hash.restype = u64
    L.oracle_u64_hash.argtypes = [p, u64]
    L.oracle_read_sums.argtypes = [u64] * 9 + [u64, p, u64]
    L.oracle_read_sums.argtypes = [u64, u64, u64, u64, u64, u64, u64, u64, u64, p, u64]
    L.oracle_write_copy_sinks.argtypes = [u64, u64, u64, u64, u64, u64, u64, C.c_int, p, u64]
    L.oracle_copy_vector_sinks.argtypes = [u64, u64, u64, u64, u64, u64, u64, p, u64]
    L.oracle_control_sinks.argtypes = [u64, p, u64]
    L.oracle_chase_links.argtypes = [u64, u64, p]
    L.oracle_chase_terminal.restype = u64
    L.oracle_chase_terminal.argtypes = [p, u64, u64, u64, u64]
    L.oracle_sfu_initial_bits.restype = C.c_uint32
    L.oracle_sfu_initial_bits.argtypes = [u64, u64, C.c_int]
    L.oracle_sfu_uniform_bits.restype = C.c_uint32
    L.oracle_sfu_uniform_bits.argtypes = [u64, u64, C.c_int]
    L.oracle_lcg_words.argtypes = [u64, u64, p]
    L.oracle_read_sums_of.argtypes = [p] + [u64] * 8 + [p, u64]
    return L


def lcg_words(n: int, seed: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.uint32)
    lib().oracle_lcg_words(n, seed, out.ctypes.data)
    return out


def read_sums_of(payload: np.ndarray, words, offset_words, blocks, threads, stride, iterations, slice_words=0, unit=1,
                 count=None):
    count = blocks * threads if count is None else count
    buf = np.ascontiguousarray(payload, dtype=np.uint32)
    out = np.zeros(count, dtype=np.uint32)
    lib().oracle_read_sums_of(buf.ctypes.data, words, offset_words, blocks, threads, stride, iterations, slice_words,
                              unit, out.ctypes.data, count)
    return out


def sfu_uniform_bits(lane: int, seed: int, chain: int) -> int:
    return int(lib().oracle_sfu_uniform_bits(lane, seed, chain))


def sink_hash(words: np.ndarray) -> int:
    w = np.ascontiguousarray(words, dtype=np.uint32)
    return int(lib().oracle_sink_hash(w.ctypes.data, w.size))


def read_sums(words, offset_words, seed, blocks, threads, stride, iterations, slice_words=0, unit=1, count=None):
    count = blocks * threads if count is None else count
    out = np.zeros(count, dtype=np.uint32)
    lib().oracle_read_sums(words, offset_words, seed, blocks, threads, stride, iterations, slice_words, unit,
                           out.ctypes.data, count)
    return out


def write_copy_sinks(words, offset_words, seed, blocks, threads, stride, iterations, copy, count=None):
    count = blocks * threads if count is None else count
    out = np.zeros(count, dtype=np.uint32)
    lib().oracle_write_copy_sinks(words, offset_words, seed, blocks, threads, stride, iterations, int(copy),
                                  out.ctypes.data, count)
    return out


def copy_vector_sinks(quads, offset_words, seed, blocks, threads, stride, iterations, count=None):
    count = blocks * threads if count is None else count
    out = np.zeros(count, dtype=np.uint32)
    lib().oracle_copy_vector_sinks(quads, offset_words, seed, blocks, threads, stride, iterations, out.ctypes.data, count)
    return out


def control_sinks(iterations, count):
    out = np.zeros(count, dtype=np.uint32)
    lib().oracle_control_sinks(iterations, out.ctypes.data, count)
    return out


def chase_links(nodes, seed):
    out = np.zeros(nodes, dtype=np.uint32)
    lib().oracle_chase_links(nodes, seed, out.ctypes.data)
    return out


def chase_terminal(links, iterations, nonce, block):
    return int(lib().oracle_chase_terminal(links.ctypes.data, links.size, iterations, nonce, block))
