"""The Nsight CSV reader and unit normaliser against the reference's (CPU)."""
from __future__ import annotations

import math

import pytest

from conftest import load_golden
from profiling_cases import CELLS, CSV_TEXTS
from powermodeling_b200 import profiling as P

GOLDEN = load_golden("profiling.json.gz")


def test_counter_list_is_the_references():
    assert P.METRICS == GOLDEN["metrics"]


def _same(a, b):
    if isinstance(a, float) and isinstance(b, float):
        return a == b or (math.isnan(a) and math.isnan(b))
    return a == b


def test_cells_normalise_as_the_reference():
    assert [[v, u] for v, u, _ in GOLDEN["cells"]] == [[v, u] for v, u in CELLS]
    for value, unit, want in GOLDEN["cells"]:
        got = list(P.normalize_metric_value(value, unit))
        assert all(_same(x, y) for x, y in zip(got, want)), (value, unit, got, want)


@pytest.mark.parametrize("index", range(len(CSV_TEXTS)))
def test_csv_logs_parse_as_the_reference(index):
    want = GOLDEN["texts"][index]
    if "error" in want:
        with pytest.raises(ValueError, match=want["error"]):
            P.parse_ncu_csv(CSV_TEXTS[index])
    else:
        assert P.parse_ncu_csv(CSV_TEXTS[index]) == want["rows"]


def test_profile_command_captures_the_target_kernel_without_clock_control():
    argv = ["--workload", "hbm", "--blocks", 1184]
    command = P.profile_command("ncu", argv, "hbm", 2, available={P.DRAM_READ, P.DURATION, "other__metric"},
                                log_file="x.csv")
    assert command[:3] == ["ncu", "--devices", "2"] and command[-4:] == ["--workload", "hbm", "--blocks", "1184"]
    assert command[command.index("--clock-control") + 1] == "none"
    assert command[command.index("--metrics") + 1] == f"{P.DRAM_READ},{P.DURATION}"
    assert "read_vector_kernel" in command[command.index("--kernel-name") + 1]
    assert "--kernel-name" not in P.profile_command("ncu", [], "gemm")
    with pytest.raises(ValueError):
        P.profile_command("ncu", [], "hbm", available=set())
    rows = P.parse_ncu_csv(CSV_TEXTS[0])
    counters = P.launch_counters(rows)
    assert counters[("0", "read_vector_kernel(...)")][P.DRAM_READ] == 4294967296.0
    assert counters[("1", "tensor_mma_kernel<2>(...)")]["sm__inst_executed_pipe_tensor.sum"] is None
