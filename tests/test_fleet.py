"""Fleet arm bookkeeping on CPU: per-GPU rows summed per rate."""
from __future__ import annotations

from powermodeling_b200 import fleet


def test_fleet_summary_sums_rates_per_key():
    rows = [{"device": 0, "throughput_bytes_s": 7.0e12, "sm_mhz": 1965},
            {"device": 1, "throughput_bytes_s": 6.9e12, "throughput_ops_s": None},
            {"device": 2, "throughput_ops_s": 2.0}]
    s = fleet.fleet_summary(rows, wall_s=1.5)
    assert s["gpus"] == 3 and s["wall_s"] == 1.5 and s["per_gpu"] is rows
    assert s["throughput_bytes_s"] == {"sum": 13.9e12, "min": 6.9e12, "max": 7.0e12}
    assert s["throughput_ops_s"] == {"sum": 2.0, "min": 2.0, "max": 2.0}
    assert "throughput_elements_s" not in s


def test_cli_requires_the_separator():
    import pytest
    with pytest.raises(SystemExit):
        fleet.main(["--gpus", "2"])
