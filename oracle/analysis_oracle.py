"""Oracle (test infrastructure only): a CPU restatement of the reference's analysis numerics.

Nothing in the product imports this module; the tests, ``__graft_entry__.smoke``
and ``bench.py``'s CPU baseline use it as the checker.  It restates, in plain
Python over the runner's trial dicts, the reference's algorithm in
powermodeling/analysis.py:
  samples/interpolate/integrate   analysis.py:85-124
  phase_stats                     analysis.py:127-207
  idle_at                         analysis.py:210-216
  measure_epochs                  analysis.py:228-276
  analyze_trial numeric body      analysis.py:597-1056 (values, validity gates)
  paired contrast                 analysis.py:292-423
  median_ci                       analysis.py:1096-1101 (generalised to B draws)
  group medians                   analysis.py:1455-1470
  nonlinear element energies      analysis.py:1027-1041 (count contract: nonlinear_oracle)
Arithmetic follows the reference operation by operation with CPython's own
float semantics (sum() is CPython 3.12's compensated sum, statistics.median,
random.Random), so the oracle's numbers equal the reference's.  The oracle is
pinned against the reference's outputs by tests/golden (see make_golden.py).
"""
from __future__ import annotations

import math
import random
import statistics

from .nonlinear_oracle import count_issues as nonlinear_count_issues

TENSOR = {"tensor", "fp16_tensor", "tensor_fp16", "gemm"}
MEMORY = {"l1", "l2", "hbm"}
SFU = {"sfu_ex2", "sfu_lg2", "sfu_rcp", "sfu_rsqrt", "sfu_sqrt", "sfu_tanh"}
NONLINEAR = {"exp", "tanh", "silu", "rmsnorm", "softmax"}
ENERGY = TENSOR | MEMORY | SFU | NONLINEAR
DEFAULT_POLICY = dict(trim_s=2.0, idle_trim_s=1.0, min_measure_s=5.0, min_idle_s=4.0, min_samples=4,
                      max_sample_gap_s=2.5, clock_tolerance_fraction=0.03, max_clock_drift_fraction=0.03,
                      max_temperature_drift_c=5.0, max_idle_drift_fraction=0.10, counter_disagreement_fraction=0.10)


def num(v):
    """None for bools, non-numbers and non-finite values; float otherwise."""
    if isinstance(v, bool):
        return None
    try:
        f = float(v)
    except (TypeError, ValueError):
        return None
    return f if math.isfinite(f) else None


def med(values):
    xs = [x for v in values if (x := num(v)) is not None]
    return statistics.median(xs) if xs else None


def timeline(phase):
    keyed = {}
    for s in phase.get("samples", []):
        if isinstance(s, dict):
            t = num(s.get("t_s"))
            if t is not None:
                keyed[t] = s
    return [keyed[t] for t in sorted(keyed)]


def value_at(series, key, t):
    """Linear value of field `key` at time t, None outside coverage or next to a gap in values."""
    if not series or t < float(series[0]["t_s"]) or t > float(series[-1]["t_s"]):
        return None
    prev = None
    for s in series:
        ts = float(s["t_s"])
        if ts == t:
            return num(s.get(key))
        if ts > t:
            a, b = num(prev.get(key)), num(s.get(key))
            if a is None or b is None:
                return None
            w = (t - float(prev["t_s"])) / (ts - float(prev["t_s"]))
            return a + w * (b - a)
        prev = s
    return None


def trapezoid(series, key, start, end):
    lo, hi = value_at(series, key, start), value_at(series, key, end)
    if lo is None or hi is None or end <= start:
        return None
    pts = [(start, lo)]
    for s in series:
        t = float(s["t_s"])
        if start < t < end:
            v = num(s.get(key))
            if v is None:
                return None
            pts.append((t, v))
    pts.append((end, hi))
    return sum((q[0] - p[0]) * (p[1] + q[1]) * 0.5 for p, q in zip(pts, pts[1:]))


def phase_stats(phase, name, pol):
    out = {"name": name, "issues": [], "warnings": []}
    if not phase:
        out["issues"].append(f"missing_phase:{name}")
        return out
    idle = name.startswith("idle_")
    a, b = num(phase.get("start_s")), num(phase.get("end_s"))
    trim = pol["idle_trim_s"] if idle else pol["trim_s"]
    if a is None or b is None or b <= a or b - a <= trim * 2:
        out["issues"].append(f"invalid_phase_window:{name}")
        return out
    a, b = a + trim, b - trim
    dur = b - a
    series = timeline(phase)
    sel = [s for s in series if a <= float(s["t_s"]) <= b]
    before = [s for s in series if float(s["t_s"]) < a][-1:]
    after = [s for s in series if float(s["t_s"]) > b][:1]
    cover = before + sel + after
    gaps = [float(y["t_s"]) - float(x["t_s"]) for x, y in zip(cover, cover[1:])]
    out.update(start_s=a, end_s=b, duration_s=dur, midpoint_s=(a + b) / 2, samples=len(sel),
               sample_interval_median_s=med(gaps), max_sample_gap_s=max(gaps) if gaps else None)
    if dur + 1e-9 < (pol["min_idle_s"] if idle else pol["min_measure_s"]):
        out["issues"].append(f"short_plateau:{name}")
    if len(sel) < pol["min_samples"]:
        out["issues"].append(f"too_few_samples:{name}")
    if gaps and max(gaps) > pol["max_sample_gap_s"]:
        out["issues"].append(f"telemetry_gap:{name}")
    energy = trapezoid(cover, "power_w", a, b)
    if any((v := num(s.get("power_w"))) is not None and v < 0 for s in cover):
        out["issues"].append(f"negative_power:{name}")
    out["integrated_power_energy_j"] = energy
    out["integrated_power_w"] = energy / dur if energy is not None else None
    out["power_w"] = out["integrated_power_w"]
    if energy is None:
        out["issues"].append(f"missing_power_coverage:{name}")
    mem = trapezoid(cover, "memory_power_w", a, b)
    out["memory_rail_energy_j"] = mem
    out["memory_power_w"] = mem / dur if mem is not None else None
    anchor = 0
    for s in cover:
        if type(s.get("energy_mj")) is int:
            anchor = s["energy_mj"]
            break
    rel = []
    for s in cover:
        c = s.get("energy_mj")
        ok = isinstance(c, (int, float)) and not isinstance(c, bool) and c >= 0
        rel.append({"t_s": s["t_s"], "r": c - anchor if ok else None})
    c0, c1 = value_at(rel, "r", a), value_at(rel, "r", b)
    present = [x for r in rel if (x := num(r["r"])) is not None]
    reset = any(y < x for x, y in zip(present, present[1:]))
    counter = None
    if c0 is not None and c1 is not None:
        if reset or c1 < c0:
            out["warnings"].append(f"energy_counter_reset:{name}")
        else:
            counter = (c1 - c0) / 1000.0
    out["energy_counter_j"] = counter
    if counter is not None:
        out["power_w"] = counter / dur
    if counter is not None and energy is not None and energy > 0:
        d = abs(counter - energy) / energy
        out["counter_power_disagreement_fraction"] = d
        if d > pol["counter_disagreement_fraction"]:
            out["issues"].append(f"energy_counter_disagreement:{name}")
    powers = [num(s.get("power_w")) for s in sel]
    changes = [float(y["t_s"]) for x, y in zip(sel, sel[1:]) if num(x.get("power_w")) != num(y.get("power_w"))]
    out["distinct_power_values"] = len({p for p in powers if p is not None})
    out["observed_power_change_interval_median_s"] = med([y - x for x, y in zip(changes, changes[1:])])
    for key in ("graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz", "temperature_c"):
        vs = [x for s in sel if (x := num(s.get(key))) is not None]
        out[key] = statistics.median(vs) if vs else None
        out[key + "_min"] = min(vs) if vs else None
        out[key + "_max"] = max(vs) if vs else None
    out["_selected"] = sel
    return out


def idle_at(pre, post, act, key):
    a, b = num(pre.get(key)), num(post.get(key))
    t0, t1, t = num(pre.get("midpoint_s")), num(post.get("midpoint_s")), num(act.get("midpoint_s"))
    if None in (a, b, t0, t1, t) or t1 <= t0 or not t0 <= t <= t1:
        return None
    return a + (b - a) * (t - t0) / (t1 - t0)


def measure_epochs(bench, phase, pol):
    src = bench.get("measure_epochs", bench.get("work_epochs"))
    if src is None:
        return [], []
    if not isinstance(src, list) or not src:
        return [], ["invalid_measure_epochs"]
    a, b = num(phase.get("start_s")), num(phase.get("end_s"))
    if a is None or b is None:
        return [], ["invalid_measure_epochs_phase_window"]
    rows = []
    for e in src:
        if not isinstance(e, dict):
            return [], ["invalid_measure_epoch"]
        x, y = num(e.get("start_s")), num(e.get("end_s"))
        if x is None:
            st = num(e.get("host_monotonic_start_ns", e.get("start_ns")))
            x = st / 1e9 if st is not None else None
        if y is None:
            st = num(e.get("host_monotonic_end_ns", e.get("end_ns")))
            y = st / 1e9 if st is not None else None
        if x is None or y is None or y <= x or x < a - 1e-6 or y > b + 1e-6:
            return [], ["invalid_measure_epoch_boundaries"]
        for k in ("operations", "logical_bytes"):
            c = num(e.get(k))
            if c is None or c < 0:
                return [], [f"invalid_measure_epoch_count:{k}"]
        rows.append({**e, "start_s": x, "end_s": y, "operations": num(e["operations"]),
                     "logical_bytes": num(e["logical_bytes"])})
    rows.sort(key=lambda e: e["start_s"])
    if any(q["start_s"] < p["end_s"] - 1e-6 for p, q in zip(rows, rows[1:])):
        return [], ["overlapping_measure_epochs"]
    inner = [e for e in rows if e["start_s"] >= a + pol["trim_s"] - 1e-6 and e["end_s"] <= b - pol["trim_s"] + 1e-6]
    if not inner or inner[-1]["end_s"] - inner[0]["start_s"] < pol["min_measure_s"] - 1e-6:
        return [], ["insufficient_complete_measure_epochs"]
    for k in ("operations", "logical_bytes"):
        whole = num(bench.get(k))
        counted = sum(e[k] for e in rows)
        if whole is not None and abs(counted - whole) > max(abs(whole) * 1e-6, 1.0):
            return [], [f"measure_epoch_total_disagreement:{k}"]
    return inner, []


def phases_of(record):
    p = record.get("phases", {})
    if isinstance(p, list):
        p = {x["name"]: x for x in p if isinstance(x, dict) and "name" in x}
    return p


def analyze(record, policy=None):
    """Numeric body of analyze_trial: the values the kernels compute, plus validity."""
    pol = dict(DEFAULT_POLICY, **(policy or {}))
    bench = record.get("benchmark") or record.get("result") or {}
    ph = phases_of(record)
    stats = {n: phase_stats(ph.get(n), n, pol) for n in ("idle_pre", "measure", "idle_post")}
    epochs, ep_issues = measure_epochs(bench, ph.get("measure") or {}, pol)
    if epochs:
        stats["measure"] = phase_stats({**ph["measure"], "start_s": epochs[0]["start_s"], "end_s": epochs[-1]["end_s"]},
                                       "measure", dict(pol, trim_s=0))
    if ph.get("active_control"):
        stats["active_control"] = phase_stats(ph["active_control"], "active_control", pol)
    m, pre, post = stats["measure"], stats["idle_pre"], stats["idle_post"]
    workload = record.get("workload")
    idle = idle_at(pre, post, m, "power_w")
    dur = num(m.get("duration_s"))
    total = num(m.get("energy_counter_j"))
    source = "energy_counter_delta"
    if total is None:
        total, source = num(m.get("integrated_power_energy_j")), "power_trapezoid"
    board = total / dur if total is not None and dur and dur > 0 else None
    idle_e = idle * dur if idle is not None and dur else None
    inc = total - idle_e if total is not None and idle_e is not None else None
    dev = num(bench.get("duration_s"))
    meas = num(bench.get("host_duration_s")) or dev
    ops, byts = num(bench.get("operations")), num(bench.get("logical_bytes"))
    ops_rate = ops / meas if ops is not None and meas and meas > 0 else None
    byte_rate = byts / meas if byts is not None and meas and meas > 0 else None
    exact = bool(epochs) and all(e.get("counts_exact") is True for e in epochs)
    c_ops = sum(e["operations"] for e in epochs) if epochs else None
    c_bytes = sum(e["logical_bytes"] for e in epochs) if epochs else None
    if epochs and dur and dur > 0:
        ops_rate, byte_rate = c_ops / dur, c_bytes / dur
    inc_p = inc / dur if inc is not None and dur else None
    ok_ops = bool(ops_rate and ops_rate > 0)
    ok_bytes = bool(byte_rate and byte_rate > 0)
    out = {"duration_s": dur, "total_energy_j": total, "energy_source": source, "board_power_w": board,
           "idle_power_w": idle, "idle_energy_j": idle_e, "incremental_energy_j": inc, "incremental_power_w": inc_p,
           "throughput_ops_s": ops_rate, "throughput_bytes_s": byte_rate,
           "counted_measure_operations": c_ops, "counted_measure_logical_bytes": c_bytes,
           "count_energy_time_alignment_exact": exact, "epoch_issues": ep_issues,
           "pj_per_op": inc_p / ops_rate * 1e12 if inc_p is not None and ok_ops and workload in ENERGY else None,
           "total_pj_per_op": board / ops_rate * 1e12 if board is not None and ok_ops and workload in ENERGY else None,
           "pj_per_logical_byte": inc_p / byte_rate * 1e12 if inc_p is not None and ok_bytes else None,
           "total_pj_per_flop": board / ops_rate * 1e12 if workload in TENSOR and board is not None and ok_ops else None,
           "operational_idle_increment_pj_per_flop": inc_p / ops_rate * 1e12 if workload in TENSOR and inc_p is not None and ok_ops else None,
           "total_pj_per_logical_bit": board / byte_rate / 8 * 1e12 if workload in MEMORY and board is not None and ok_bytes else None,
           "operational_idle_increment_pj_per_logical_bit": inc_p / byte_rate / 8 * 1e12 if workload in MEMORY and inc_p is not None and ok_bytes else None,
           "phases": {k: {x: y for x, y in v.items() if not x.startswith("_")} for k, v in stats.items()}}
    sel = m.get("_selected", [])
    limit = med(s.get("power_limit_w") for s in sel)
    if not limit:
        device, config = record.get("device") or {}, dict(record.get("config") or {})
        limit = (num(record.get("power_limit_w", device.get("power_limit_w", config.get("power_limit_w"))))
                 or num((device.get("sample") or {}).get("power_limit_w")))
    out.update(graphics_clock_mhz=m.get("graphics_clock_mhz"), sm_clock_mhz=m.get("sm_clock_mhz"),
               memory_clock_mhz=m.get("memory_clock_mhz"), temperature_c=m.get("temperature_c"), power_limit_w=limit,
               operational_idle_increment_power_w=inc_p, operational_idle_increment_energy_j=inc,
               idle_fraction_of_measured_power=idle / board if idle is not None and board and board > 0 else None,
               idle_fraction_of_power_limit=idle / limit if idle is not None and limit and limit > 0 else None,
               power_limit_utilization=board / limit if board is not None and limit and limit > 0 else None,
               memory_rail_power_w=m.get("memory_power_w"),
               total_pj_per_logical_byte=board / byte_rate * 1e12 if board is not None and ok_bytes else None)
    # paired reference
    ref_phase = ph.get("active_reference")
    if ref_phase:
        ref_rec = record.get("active_reference") or {}
        ref = phase_stats(ref_phase, "active_reference", pol)
        r_epochs, r_issues = measure_epochs(ref_rec, ref_phase, pol)
        if r_epochs:
            ref = phase_stats({**ref_phase, "start_s": r_epochs[0]["start_s"], "end_s": r_epochs[-1]["end_s"]},
                              "active_reference", dict(pol, trim_s=0))
        rp = num(ref.get("power_w"))
        contrast = board - rp if board is not None and rp is not None else None
        out.update(active_reference_power_w=rp, paired_active_reference_power_w=contrast,
                   paired_active_reference_energy_j=contrast * dur if contrast is not None and dur else None,
                   active_reference_duration_s=ref.get("duration_s"),
                   paired_active_reference_pj_per_flop=contrast / ops_rate * 1e12 if workload in TENSOR and contrast is not None and ok_ops else None,
                   paired_active_reference_pj_per_logical_bit=contrast / byte_rate / 8 * 1e12 if workload in MEMORY and contrast is not None and ok_bytes else None,
                   reference_epoch_issues=r_issues)
        out["phases"]["active_reference"] = {x: y for x, y in ref.items() if not x.startswith("_")}
    # complete nonlinear functions: per-element and per-row energies (analysis.py:1027-1041)
    nonlinear = workload in NONLINEAR
    contract_ok = nonlinear and not nonlinear_count_issues(bench, workload)
    element_rate = ops_rate if contract_ok and exact and ops_rate and ops_rate > 0 else None
    width = bench.get("row_width") if workload in ("rmsnorm", "softmax") else None
    row_rate = element_rate / width if element_rate and width else None
    out.update(throughput_elements_s=element_rate, throughput_rows_s=row_rate,
               row_width=bench.get("row_width") if nonlinear else None,
               counted_measure_elements=c_ops if element_rate else None)
    if nonlinear and element_rate is None:
        out["pj_per_op"] = out["total_pj_per_op"] = None
    for prefix, power in (("total_", board), ("operational_idle_increment_", inc_p),
                          ("paired_active_reference_", out.get("paired_active_reference_power_w"))):
        out[prefix + "pj_per_element"] = power / element_rate * 1e12 if power is not None and element_rate else None
        out[prefix + "pj_per_row"] = power / row_rate * 1e12 if power is not None and row_rate else None
    return out


def median_ci(values, seed, resamples=1000):
    """_median_ci generalised to `resamples` draws; B=1000 is the reference exactly."""
    if len(values) < 3:
        return None
    rng = random.Random(seed)
    draws = sorted(statistics.median(rng.choices(values, k=len(values))) for _ in range(resamples))
    return [draws[25 * resamples // 1000 - 1], draws[975 * resamples // 1000 - 1]]


def resample_indices(seed, n, resamples):
    """The index stream choices() draws: rows of floor(random()*n)."""
    rng = random.Random(seed)
    idx = list(range(n))
    return [rng.choices(idx, k=n) for _ in range(resamples)]


METRICS = ("board_power_w", "idle_power_w", "incremental_power_w", "throughput_ops_s", "throughput_bytes_s",
           "pj_per_op", "pj_per_logical_byte", "total_pj_per_op", "total_pj_per_logical_byte",
           "memory_rail_power_w", "memory_rail_incremental_power_w", "graphics_clock_mhz", "sm_clock_mhz",
           "memory_clock_mhz", "temperature_c", "idle_fraction_of_measured_power", "idle_fraction_of_power_limit",
           "power_limit_utilization", "tensor_peak_tflops_at_achieved_clock", "tensor_utilization_vs_dense_clock_peak",
           "total_pj_per_flop", "total_pj_per_logical_bit", "operational_idle_increment_power_w",
           "operational_idle_increment_energy_j", "operational_idle_increment_pj_per_flop",
           "operational_idle_increment_pj_per_logical_bit", "paired_active_reference_power_w",
           "paired_active_reference_energy_j", "paired_active_reference_pj_per_flop",
           "paired_active_reference_pj_per_logical_bit", "throughput_elements_s", "throughput_rows_s",
           "total_pj_per_element", "total_pj_per_row", "operational_idle_increment_pj_per_element",
           "operational_idle_increment_pj_per_row", "paired_active_reference_pj_per_element",
           "paired_active_reference_pj_per_row", "throughput_sfu_instructions_s", "total_pj_per_instruction",
           "operational_idle_increment_pj_per_instruction", "paired_active_reference_pj_per_instruction",
           "sfu_reference_delta_pj_per_instruction", "sfu_reference_delta_power_w", "active_reference_duration_s",
           "active_reference_counted_loop_slots", "active_reference_loop_slots_s")


def group_summary(records, seed, policy=None, resamples=1000):
    """Medians and intervals of every _METRICS entry over one group's trials (all assumed valid)."""
    rows = [analyze(r, policy) for r in records]
    return group_medians_and_cis([[row.get(m) for m in METRICS] for row in rows], seed, resamples)


def group_medians_and_cis(rows, seed, resamples=1000):
    """Per metric column: (median, ci) over the finite entries of `rows` in order."""
    out = []
    for col in zip(*rows):
        vals = [x for v in col if (x := num(v)) is not None]
        out.append((statistics.median(vals) if vals else None, median_ci(vals, seed, resamples)))
    return out
