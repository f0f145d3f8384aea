"""Dense FP16 tensor issue capacity per SM per clock, by compute capability.

The reference's table (powermodeling/profiles.py:9-13) covers V100, A100 and
H100 and rejects any other device.  B200 (compute capability 10.0) is added
here: tcgen05 issues a dense FP16 MMA at twice Hopper's per-SM rate, 8192
FLOP/SM/clock (2.25 PFLOP/s dense at 148 SMs and about 1.86 GHz).  The
value is a datasheet figure, not a measurement; the tensor workload reports
achieved TFLOP/s beside it.
"""

ARCHITECTURES = {
    (7, 0): {"architecture": "Volta", "family": "V100", "dense_tensor_flops_per_sm_clock": 1024},
    (8, 0): {"architecture": "Ampere GA100", "family": "A100", "dense_tensor_flops_per_sm_clock": 2048},
    (9, 0): {"architecture": "Hopper", "family": "H100", "dense_tensor_flops_per_sm_clock": 4096},
    (10, 0): {"architecture": "Blackwell GB100", "family": "B200", "dense_tensor_flops_per_sm_clock": 8192},
}


def theoretical_tensor_tflops(flops_per_sm_clock: int, sm_count: int, clock_mhz: float) -> float:
    """Clock-specific dense ceiling, in the reference's operation order (profiles.py:94-98)."""
    return flops_per_sm_clock * sm_count * clock_mhz * 1e6 / 1e12
