"""ctypes binding of libpmb200 (include/pmb200.h).

The library is built in tree (``python -m powermodeling_b200.build``) and
loaded from this package directory.  There is no fallback: when the library
is missing or no CUDA device is visible, every compute entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import numpy as np

LIBRARY = Path(__file__).resolve().parent / "libpmb200.so"

PM_OK = 0
PM_PHASES = 5
PHASE_NAMES = ("idle_pre", "measure", "idle_post", "active_reference", "active_control")
WL_OTHER, WL_TENSOR, WL_MEMORY, WL_SFU, WL_NONLINEAR = range(5)

# sample flags
S_THROTTLE_VALID = 0x0001
S_FOREIGN_PID = 0x0002
S_NO_COMPUTE_INV = 0x0004
S_NO_GRAPHICS_INV = 0x0008
S_MPS = 0x0010
S_PID_UNKNOWN = 0x0020
S_ENERGY_ANCHOR = 0x0040
S_ENERGY_INT = 0x0080
S_ENERGY_FLOAT = 0x0100
S_REF_FOREIGN = 0x0200
S_MEMORY_POWER_SET = 0x0400
# trial flags
T_HOST_ISSUES = 0x0008
T_HOST_BASELINE = 0x0010
T_HOST_PAIRED = 0x0020
T_ORDER_AB = 0x0040
T_ORDER_BA = 0x0080
T_TENSOR_PEAK_KNOWN = 0x0100
T_SFU_CONTRACT_OK = 0x0200
T_NONLINEAR_OK = 0x0400
T_ROWWISE = 0x0800
# epoch list status
EP_NONE, EP_OK, EP_INVALID_LIST, EP_NON_DICT_AFTER = range(4)
# trial scalar slots
TS = dict(BENCH_DURATION_S=0, BENCH_HOST_DURATION_S=1, BENCH_OPERATIONS=2, BENCH_LOGICAL_BYTES=3,
          REF_OPERATIONS=4, REF_LOGICAL_BYTES=5, REQ_GRAPHICS_MHZ=6, REQ_MEMORY_MHZ=7, REQ_SM_MHZ=8,
          TENSOR_FLOPS_PER_CLOCK=9, POWER_LIMIT_FALLBACK_W=10, ROW_WIDTH=11)
TS_COUNT = 12

_p = C.c_void_p


class Policy(C.Structure):
    _fields_ = [("trim_s", C.c_double), ("idle_trim_s", C.c_double), ("min_measure_s", C.c_double),
                ("min_idle_s", C.c_double), ("min_samples", C.c_int32), ("max_sample_gap_s", C.c_double),
                ("clock_tolerance_fraction", C.c_double), ("max_clock_drift_fraction", C.c_double),
                ("max_temperature_drift_c", C.c_double), ("max_idle_drift_fraction", C.c_double),
                ("counter_disagreement_fraction", C.c_double)]


TRIAL_ARRAYS = (
    # (name, dtype, length key)
    ("phase_offsets", np.int64, "slots+1"), ("phase_start_s", np.float64, "slots"),
    ("phase_end_s", np.float64, "slots"), ("phase_present", np.uint8, "slots"),
    ("t_s", np.float64, "samples"), ("power_w", np.float64, "samples"), ("memory_power_w", np.float64, "samples"),
    ("graphics_clock_mhz", np.float64, "samples"), ("sm_clock_mhz", np.float64, "samples"),
    ("memory_clock_mhz", np.float64, "samples"), ("temperature_c", np.float64, "samples"),
    ("power_limit_w", np.float64, "samples"), ("enforced_power_limit_w", np.float64, "samples"),
    ("pstate", np.float64, "samples"), ("energy_int", np.int64, "samples"), ("energy_float", np.float64, "samples"),
    ("throttle_reasons", np.int64, "samples"), ("sample_flags", np.uint16, "samples"),
    ("memory_power_source", np.uint8, "samples"),
)
EPOCH_ARRAYS = (
    ("epoch_offsets", np.int32, "arms+1"), ("epoch_status", np.int32, "arms"),
    ("epoch_start_s", np.float64, "epochs"), ("epoch_end_s", np.float64, "epochs"),
    ("epoch_operations", np.float64, "epochs"), ("epoch_logical_bytes", np.float64, "epochs"),
    ("epoch_loop_slots", np.float64, "epochs"), ("epoch_counts_exact", np.uint8, "epochs"),
)
TAIL_ARRAYS = (("trial_scalars", np.float64, "scalars"), ("trial_flags", np.uint32, "trials"))


class Trials(C.Structure):
    _fields_ = ([("n_trials", C.c_int32), ("max_phase_samples", C.c_int32), ("n_samples", C.c_int64)]
                + [(name, _p) for name, _, _ in TRIAL_ARRAYS]
                + [("n_epochs", C.c_int32)]
                + [(name, _p) for name, _, _ in EPOCH_ARRAYS + TAIL_ARRAYS]
                + [("broadcast_columns", C.c_uint32)])


# Per-sample columns that the packer may broadcast, with their PM_COL_* bit.
BROADCAST_COLUMNS = (("power_w", 1 << 0), ("memory_power_w", 1 << 1), ("graphics_clock_mhz", 1 << 2),
                     ("sm_clock_mhz", 1 << 3), ("memory_clock_mhz", 1 << 4), ("temperature_c", 1 << 5),
                     ("power_limit_w", 1 << 6), ("enforced_power_limit_w", 1 << 7), ("pstate", 1 << 8),
                     ("energy_int", 1 << 9), ("energy_float", 1 << 10), ("throttle_reasons", 1 << 11),
                     ("sample_flags", 1 << 12), ("memory_power_source", 1 << 13))


class TrialResults(C.Structure):
    _fields_ = [("phase_out", _p), ("phase_flags", _p), ("trial_out", _p), ("issue_bits", _p),
                ("metrics", _p), ("valid", _p)]


class BootstrapJob(C.Structure):
    _fields_ = [("n_groups", C.c_int32), ("n_metrics", C.c_int32), ("n_members", C.c_int32),
                ("n_rows", C.c_int32), ("resamples", C.c_int32), ("max_members", C.c_int32),
                ("values", _p), ("group_offsets", _p), ("member_rows", _p), ("member_valid", _p),
                ("seeds", _p), ("medians", _p), ("ci_lo", _p), ("ci_hi", _p)]


MAX_RANKS = 8   # PM_MAX_RANKS (include/pmb200_peer.h)


class PeerHandle(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64)]


class PeerRows(C.Structure):
    _fields_ = [("n_ranks", C.c_int32), ("rank", C.c_int32), ("row_offset", C.c_int32), ("epoch", C.c_uint32),
                ("metrics", _p * MAX_RANKS), ("valid", _p * MAX_RANKS), ("flags", _p * MAX_RANKS), ("done", _p)]


class PeerGroups(C.Structure):
    _fields_ = [("n_ranks", C.c_int32), ("rank", C.c_int32), ("per_rank", C.c_int32), ("epoch", C.c_uint32),
                ("out", _p * MAX_RANKS), ("flags", _p * MAX_RANKS), ("done", _p), ("root", C.c_int32)]


class NativeError(RuntimeError):
    """A libpmb200 entry point returned an error code."""


_lock = threading.Lock()
_lib = None


def library() -> C.CDLL:
    """Load libpmb200 once; raise if it is absent (there is no CPU path)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise NativeError(f"{LIBRARY} is not built; run python -m powermodeling_b200.build")
            lib = C.CDLL(str(LIBRARY), mode=os.RTLD_NOW | getattr(os, "RTLD_GLOBAL", 0))
            lib.pm_layout.restype = C.c_int32
            lib.pm_layout.argtypes = [C.c_char_p]
            lib.pm_last_error.restype = C.c_size_t
            lib.pm_last_error.argtypes = [C.c_char_p, C.c_size_t]
            lib.pm_abi_version.restype = C.c_int32
            lib.pm_device_count.restype = C.c_int32
            lib.pm_analyze_trials.argtypes = [C.POINTER(Trials), C.POINTER(Policy), C.POINTER(TrialResults)]
            lib.pm_analyze_trials_device.argtypes = [C.POINTER(Trials), C.POINTER(Policy), C.POINTER(TrialResults),
                                                     _p, C.c_size_t, _p]
            lib.pm_analyze_scratch_bytes.restype = C.c_size_t
            lib.pm_analyze_scratch_bytes.argtypes = [C.c_int32, C.c_int32]
            lib.pm_group_bootstrap.argtypes = [C.POINTER(BootstrapJob)]
            lib.pm_group_bootstrap_device.argtypes = [C.POINTER(BootstrapJob), _p, C.c_size_t, _p]
            lib.pm_bootstrap_prepare_device.argtypes = [C.POINTER(BootstrapJob), _p, C.c_size_t, _p]
            lib.pm_bootstrap_finish_device.argtypes = [C.POINTER(BootstrapJob), _p, C.c_size_t, _p]
            lib.pm_bootstrap_scratch_bytes.restype = C.c_size_t
            lib.pm_bootstrap_scratch_bytes.argtypes = [C.c_int32, C.c_int32, C.c_int32]
            lib.pm_analyze_sweep.argtypes = [C.POINTER(Trials), C.POINTER(Policy), C.POINTER(TrialResults),
                                             C.POINTER(BootstrapJob)]
            lib.pm_analyze_sweep_scratch_bytes.restype = C.c_size_t
            lib.pm_analyze_sweep_scratch_bytes.argtypes = [C.c_int32] * 5
            lib.pm_analyze_sweep_device.argtypes = [C.POINTER(Trials), C.POINTER(Policy), C.POINTER(TrialResults),
                                                    C.POINTER(BootstrapJob), _p, C.c_size_t, _p, _p]
            lib.pm_resample_indices.argtypes = [C.c_uint64, C.c_int32, C.c_int32, C.POINTER(C.c_int32)]
            lib.pm_peer_alloc.argtypes = [C.c_size_t, C.POINTER(_p), C.POINTER(PeerHandle)]
            lib.pm_peer_free.argtypes = [_p]
            lib.pm_peer_open.argtypes = [C.POINTER(PeerHandle), C.POINTER(_p)]
            lib.pm_peer_close.argtypes = [_p]
            lib.pm_analyze_trials_device_exchange.argtypes = [C.POINTER(Trials), C.POINTER(Policy), C.POINTER(TrialResults),
                                                              _p, C.c_size_t, C.POINTER(PeerRows), _p]
            lib.pm_peer_wait_device.argtypes = [_p, C.c_int32, C.c_uint32, C.c_uint32, _p, _p]
            lib.pm_peer_gate_device.argtypes = [C.POINTER(_p), C.c_int32, C.c_int32, C.c_uint32, C.c_uint32, _p, _p]
            lib.pm_bootstrap_finish_device_exchange.argtypes = [C.POINTER(BootstrapJob), _p, C.c_size_t,
                                                                C.POINTER(PeerGroups), _p]
            lib.pm_nonlinear_fill_device.argtypes = [_p, C.c_uint64, C.c_uint64, C.c_float, C.c_int, _p]
            lib.pm_nonlinear_apply_device.argtypes = [C.c_int32, _p, _p, _p, C.c_uint64, C.c_int32, C.c_uint64,
                                                      C.c_int32, C.c_int32, _p]
            _lib = lib
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    library().pm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != PM_OK:
        raise NativeError(f"{what} failed ({rc}): {last_error()}")


_layout_cache: dict[str, int] = {}


def layout(name: str) -> int:
    value = _layout_cache.get(name)
    if value is None:
        value = library().pm_layout(name.encode())
        if value < 0:
            raise KeyError(name)
        _layout_cache[name] = value
    return value


def ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


def resample_indices(seed: int, n: int, resamples: int) -> np.ndarray:
    out = np.empty(n * resamples, dtype=np.int32)
    check(library().pm_resample_indices(C.c_uint64(seed), n, resamples, out.ctypes.data_as(C.POINTER(C.c_int32))),
          "pm_resample_indices")
    return out.reshape(resamples, n)
