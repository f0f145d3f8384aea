"""The native record packer (_packnative) against the Python packer it replaces.

Both apply the reference's sample rules (_samples, _finite, _throttle_mask,
energy-counter kinds, process inventories, memory-power sources); every
array, the sorted sample lists and the foreign pids must be identical, and a
value the reference's coercion lets raise must raise the same exception."""
from __future__ import annotations

import copy

import numpy as np
import pytest

from powermodeling_b200 import pack as P
from powermodeling_b200.profiles import ARCHITECTURES
from powermodeling_b200.synthetic import SweepShape, make_sweep
from trial_builders import memory_rail_scenarios, scenarios


def both(records):
    flags = [0] * len(records)
    P._SOURCE_IDS.clear()
    a = P.pack_trials(records, flags, ARCHITECTURES, native=True)
    ids_a = dict(P._SOURCE_IDS)
    P._SOURCE_IDS.clear()
    b = P.pack_trials(records, flags, ARCHITECTURES, native=False)
    assert ids_a == P._SOURCE_IDS
    return a, b


def assert_same(a, b):
    assert a.arrays.keys() == b.arrays.keys()
    for k in a.arrays:
        x, y = a.arrays[k], b.arrays[k]
        assert x.dtype == y.dtype and x.shape == y.shape, k
        assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), k
    assert (a.n_trials, a.n_samples, a.n_epochs, a.max_phase_samples, a.broadcast) == \
           (b.n_trials, b.n_samples, b.n_epochs, b.max_phase_samples, b.broadcast)
    # the same sample objects in the same order (packing never copies or mutates them)
    assert [[id(x) for x in slot] for slot in a.samples] == [[id(x) for x in slot] for slot in b.samples]
    assert a.foreign_pids == b.foreign_pids


def test_scenario_records():
    records = [r for _, r, _ in scenarios()] + [r for _, r in memory_rail_scenarios()]
    assert_same(*both(records))


def test_synthetic_sweeps():
    for shape, seed in ((SweepShape(points=6, repeats=4), 3), (SweepShape(points=3, repeats=5, with_energy_counter=True), 4)):
        assert_same(*both(make_sweep(shape, seed)))


class IntLike(int):
    pass


class Floaty:
    def __float__(self):
        return 7.5


def awkward_samples():
    base = {"t_s": 0.0, "power_w": 100.0, "compute_processes": [], "graphics_processes": []}
    odd = [
        {"power_w": "123.5", "graphics_clock_mhz": True, "sm_clock_mhz": float("nan"), "memory_clock_mhz": float("inf"),
         "temperature_c": "hot", "power_limit_w": IntLike(400), "enforced_power_limit_w": Floaty(), "pstate": b"3"},
        {"energy_mj": 2 ** 63 + 5, "throttle_reasons": "0x10"},
        {"energy_mj": 2 ** 64 + 9, "throttle_reasons": "0b101"},
        {"energy_mj": -5, "throttle_reasons": "010"},
        {"energy_mj": -(2 ** 64), "throttle_reasons": "junk"},
        {"energy_mj": IntLike(12), "throttle_reasons": 2 ** 64 - 1},
        {"energy_mj": IntLike(-3), "throttle_reasons": 2 ** 64},
        {"energy_mj": 3.5, "throttle_reasons": -(2 ** 63) - 1},
        {"energy_mj": float("nan"), "throttle_reasons": float("nan")},
        {"energy_mj": float("inf"), "throttle_reasons": True},
        {"energy_mj": True, "throttle_reasons": 3.9},
        {"energy_mj": "12", "throttle_reasons": b"12"},
        {"compute_processes": [{"pid": 777}, {"pid": None}, 778, {"other": 1}], "graphics_processes": None},
        {"compute_processes": ({"pid": 1},), "graphics_processes": [777], "mps_compute_processes": [1]},
        {"mps_compute_processes": [], "memory_power_w": None, "memory_power_source": ""},
        {"memory_power_w": 0.0, "memory_power_source": "memory_power_instant_w"},
        {"memory_power_source": 17},
        {"memory_power_source": ("a", 1)},
        {"memory_power_source": "memory_power_instant_w"},
    ]
    out = []
    for k, extra in enumerate(odd):
        s = dict(base, t_s=float(k) * 0.5)
        s.update(extra)
        out.append(s)
    out += [dict(base, t_s=3.0, power_w=1.0), dict(base, t_s=3.0, power_w=2.0),        # last one wins
            dict(base, t_s=-0.0, power_w=5.0), dict(base, t_s=0.0, power_w=6.0),      # -0.0 == 0.0
            dict(base, t_s="2.25"), dict(base, t_s=IntLike(4)), "not a sample", 7, dict(base, t_s=None),
            dict(base, t_s=float("nan")), dict(base, t_s=True)]
    out.reverse()
    return out


@pytest.mark.parametrize("pid", [777, None, "777"])
def test_awkward_values(pid):
    record = [r for name, r, _ in scenarios() if name == "steady_float_counter"][0]
    record = copy.deepcopy(record)
    record["quality"]["measurement_pid"] = pid
    record["phases"]["measure"]["samples"] = awkward_samples()
    record["phases"]["idle_pre"]["samples"] = tuple(awkward_samples()[:5])
    assert_same(*both([record]))


@pytest.mark.parametrize("field,value,error", [
    ("power_w", 2 ** 2000, OverflowError),            # float() of a huge int raises (not caught by _finite)
    ("energy_mj", 2 ** 64 + 2 ** 63, OverflowError),  # still outside int64 after the 2**64 fold
    ("throttle_reasons", float("inf"), OverflowError),
])
def test_errors_the_reference_lets_raise(field, value, error):
    record = copy.deepcopy([r for name, r, _ in scenarios() if name == "steady_float_counter"][0])
    record["phases"]["measure"]["samples"][3][field] = value
    for native in (True, False):
        with pytest.raises(error):
            P.pack_trials([copy.deepcopy(record)], [0], ARCHITECTURES, native=native)


def test_fast_and_object_paths_number_sources_in_slot_order():
    """Slots packed on the parallel path and on the object-API path interleave; memory-power
    source ids still follow first sight over slots in order, as the Python packer numbers them."""
    from trial_builders import memory_rail_scenarios as rails
    records = [copy.deepcopy(r) for _, r in rails()][:4] + make_sweep(SweepShape(points=4, repeats=4), 5)
    for k, record in enumerate(records):
        for name, phase in record["phases"].items():
            for i, s in enumerate(phase.get("samples", [])):
                if isinstance(s, dict):
                    s["memory_power_source"] = ("src_a", "src_b", "memory_power_instant_w")[(k + i) % 3]
        if k % 3 == 1:      # an object the parallel path hands back to the object API
            record["phases"]["measure"]["samples"][0]["power_w"] = IntLike(3)
    a, b = both(records)
    assert_same(a, b)
    from powermodeling_b200 import _packnative
    P.pack_trials(records, [0] * len(records), ARCHITECTURES, native=True)
    assert 0 < _packnative.last_fast_slots() < 5 * len(records)


def _bits_equal(a, b) -> bool:
    """Equal with types, float bits and key order (signed zeros and NaN payloads included)."""
    import struct
    if type(a) is not type(b):
        return False
    if isinstance(a, dict):
        return list(a) == list(b) and all(_bits_equal(a[k], b[k]) for k in a)
    if isinstance(a, list):
        return len(a) == len(b) and all(_bits_equal(x, y) for x, y in zip(a, b))
    if isinstance(a, float):
        return struct.pack("<d", a) == struct.pack("<d", b)
    return a == b


def test_measure_bindings_from_the_clock_repeat_column():
    """binding_samples with the packer's clock_repeat column equals the Python statement on clocks
    that repeat, change kind (int 1 / float 1.0 / True), sign (0.0 / -0.0), go missing or None, or NaN."""
    from powermodeling_b200.trial_report import binding_samples
    rng = np.random.default_rng(5)
    records = make_sweep(SweepShape(points=4, repeats=2), 9)
    choices = [1410, 1410.0, 0.0, -0.0, None, "absent", float("nan"), True, 1, 1.0, 1980]
    for record in records:
        for phase in record["phases"].values():
            run = None
            for s in phase.get("samples", []):
                if run is None or rng.random() < 0.15:
                    run = (choices[rng.integers(len(choices))], choices[rng.integers(len(choices))])
                for key, value in zip(("graphics_clock_mhz", "memory_clock_mhz"), run):
                    if value == "absent":
                        s.pop(key, None)
                    else:
                        s[key] = value
    packed = P.pack_trials(records, [0] * len(records), ARCHITECTURES, native=True)
    assert packed.clock_repeat is not None and len(packed.clock_repeat) == packed.n_samples
    native = P._native_packer()
    offsets = packed.arrays["phase_offsets"]
    for slot, samples in enumerate(packed.samples):
        repeat = memoryview(packed.clock_repeat)[int(offsets[slot]):int(offsets[slot + 1])]
        for lo, hi in ((0, len(samples)), (3, len(samples) - 2), (len(samples) // 2, len(samples))):
            got = native.binding_samples(samples, lo, hi, repeat)
            assert _bits_equal(got, binding_samples(samples[lo:hi])), (slot, lo, hi)
            assert _bits_equal(native.binding_samples(samples, lo, hi), got)


class EpochDict(dict):
    pass


def test_epoch_lists_native_equal_python_statement():
    """Every arm shape the reference's epoch parsing distinguishes: absent, None, empty, not a list,
    measure_epochs over work_epochs (a present None included), nanosecond stamps, non-finite and
    non-numeric values, a non-dict item that stops parsing, and subclasses (the Python path)."""
    ep = lambda **kw: dict({"start_s": 1.0, "end_s": 2.0, "operations": 10, "logical_bytes": 4.5,
                            "reference_loop_slots": None, "counts_exact": True}, **kw)
    arms = [
        {}, {"measure_epochs": None}, {"measure_epochs": []}, {"measure_epochs": (ep(),)}, {"measure_epochs": "x"},
        {"work_epochs": [ep(), ep(start_s=3.0)]}, {"measure_epochs": None, "work_epochs": [ep()]},
        {"measure_epochs": [ep(start_s=None, host_monotonic_start_ns=5e9, end_s="bad", end_ns=7_000_000_000)]},
        {"measure_epochs": [ep(start_s=float("nan"), start_ns=True, end_s=float("inf"), host_monotonic_end_ns=None)]},
        {"measure_epochs": [ep(operations="12", logical_bytes=float("inf"), counts_exact=1)]},
        {"measure_epochs": [ep(), 3, ep()]}, {"measure_epochs": [ep(counts_exact=False), ep(reference_loop_slots=2 ** 70)]},
        {"measure_epochs": [EpochDict(ep()), ep()]}, EpochDict({"measure_epochs": [ep()]}),
        {"measure_epochs": [ep(start_s=True, end_s=False)]},
    ]
    a = P._epoch_columns_native(arms)
    b = P._epoch_columns_python(arms)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    for x, y in zip(a[2], b[2]):
        assert x.dtype == y.dtype and np.array_equal(x.view(np.uint8), y.view(np.uint8))
    with pytest.raises(OverflowError):
        P._epoch_columns_native([{"measure_epochs": [ep(operations=10 ** 400)]}])
