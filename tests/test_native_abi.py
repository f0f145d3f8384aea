"""The C-ABI library loads, exports what include/pmb200.h declares, and fails loudly without a GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT
from powermodeling_b200 import _native as N


def declared_functions() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(pm_\w+)\s*\(", text, flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = N.library()
    declared = declared_functions()
    assert {"pm_analyze_trials", "pm_group_bootstrap", "pm_layout", "pm_last_error"} <= declared
    missing = [name for name in sorted(declared) if not hasattr(lib, name)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIBRARY)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (pm_\w+)", out))
    assert declared <= exported, sorted(declared - exported)


def test_layout_names_resolve():
    assert N.layout("PM_PHASES") == 5
    assert N.layout("PM_M_COUNT") == 47
    assert N.layout("PM_M_board_power_w") == 0
    assert N.layout("PM_M_active_reference_loop_slots_s") == 46
    assert N.library().pm_layout(b"PM_NO_SUCH_SLOT") == -1
    assert N.library().pm_abi_version() == 1


def test_issue_tables_match_bit_counts():
    from powermodeling_b200 import analysis
    words = analysis._word_strings()
    assert [len(w) for w in words] == [N.layout(n) for n in ("PM_IT_COUNT", "PM_IB_COUNT", "PM_IP_COUNT", "PM_W_COUNT")]


def test_struct_layouts_match_header_order():
    # pm_trials: n_trials, max_phase_samples, n_samples then pointers; sizes checked against the ABI.
    assert ctypes.sizeof(N.Policy) == 11 * 8
    assert N.Trials.n_samples.offset == 8
    assert N.BootstrapJob.values.offset == 24


@pytest.mark.skipif(N.library().pm_device_count() > 0, reason="checks the no-device error path")
def test_compute_entry_points_fail_loudly_without_a_device():
    from powermodeling_b200.analysis import analyze_trials, median_ci
    from powermodeling_b200.synthetic import SweepShape, make_sweep
    with pytest.raises(N.NativeError, match="no CUDA device"):
        analyze_trials(make_sweep(SweepShape(points=1, repeats=1)))
    with pytest.raises(N.NativeError):
        median_ci([1.0, 2.0, 3.0], 5)
