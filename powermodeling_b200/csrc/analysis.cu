// Batched trial analysis on sm_100a: one CTA per trial.
//
// Restates, in data-parallel form, the numeric core of the reference's
// powermodeling/analysis.py:
//   _interpolate / _integrate            analysis.py:94-124
//   _phase_stats                         analysis.py:127-207
//   _idle_at                             analysis.py:210-216
//   _measure_epochs                      analysis.py:228-276
//   analyze_trial (numeric body, gates)  analysis.py:597-1056
//   _paired_reference_contrast           analysis.py:292-423
// Samples arrive sorted and de-duplicated per (trial, phase) slot, so the
// selection window, the covering neighbours and every interpolation bracket
// are binary searches; medians come from a CTA-wide bitonic sort of up to ten
// columns at once; the trapezoid and counter sums run sequentially on single
// lanes in the reference's order (CPython's compensated float sum), so the
// energies agree bit for bit with the reference's.
#include "pmb200.h"
#include "pm_layout.h"
#include "pm_device.cuh"
#include "pm_capi.h"
#include "pmb200_peer.h"

namespace pm {

constexpr int kThreads = 256;
constexpr int kMaxEpochs = 256;        // per arm; the host rejects longer lists
enum Col { C_GAP = 0, C_CHANGE, C_POWER, C_GFX, C_SM, C_MEM, C_TEMP, C_PLIMIT, C_ENF, C_PSTATE, C_COUNT };
// Staged covering samples that follow the sample columns in the tile.
// S_SET0/S_SET1: the distinct-power hash set (2 x SP 64-bit slots).
enum Stage { S_T = 0, S_POWER, S_MEMORY, S_REL, S_TERM_P, S_TERM_M, S_SET0, S_SET1, S_COUNT };
constexpr int kTileColumns = C_COUNT + S_COUNT;
static_assert(kTileColumns == kSortColumns, "tile column count");

struct EpochResult {
  int32_t n_inner;            // complete epochs kept (0 = none)
  int32_t issue;              // -1 none, else offset from PM_IT_EP_PHASE_WINDOW
  double start_s, end_s;      // aligned window
  double ops, bytes, slots;   // sums over kept epochs (NaN slots if any missing)
  int32_t exact;              // every kept epoch counts_exact
};

struct Shared {
  double po[PM_PHASES][PM_PO_COUNT];
  uint32_t pf[PM_PHASES];
  EpochResult ep[2];
  int16_t order[2][kMaxEpochs];
  // per-phase broadcast scratch
  int64_t sel_lo, sel_hi, cov_lo, cov_hi;
  double wstart, wend;
  int32_t nchange;
  int32_t nfin[C_COUNT];
  double cmin[C_COUNT], cmax[C_COUNT];
  int32_t med_cols[C_COUNT], nmed;   // varying columns whose median is selected (power excluded)
  double cmed[C_COUNT];              // their medians
  int32_t distinct_power;   // distinct finite powers of a varying power column, -1 if it holds one value or none
  int32_t anchor_q;         // first covering sample flagged as energy anchor (INT32_MAX: none)
};

// A read of the trial batch, which no thread writes during the launch: through
// the read-only path, so the compiler may issue it ahead of the shared-memory
// stores around it instead of after them.
template <class E>
__device__ __forceinline__ E ro(const E* p) { return __ldg(p); }
template <>
__device__ __forceinline__ int64_t ro<int64_t>(const int64_t* p) {
  return (int64_t)__ldg(reinterpret_cast<const long long*>(p));
}

// Sample i of a per-sample column; a broadcast column holds one element.
template <class E>
__device__ __forceinline__ E col_at(const E* col, uint32_t bit, const pm_trials& T, int64_t i) {
  return ro((T.broadcast_columns & bit) ? col : col + i);
}

// The PM_COL_* bit of a sample column (0: derived columns, never broadcast).
__device__ __forceinline__ uint32_t column_bit(int c) {
  switch (c) {
    case C_POWER: return PM_COL_POWER_W;
    case C_GFX: return PM_COL_GRAPHICS_CLOCK;
    case C_SM: return PM_COL_SM_CLOCK;
    case C_MEM: return PM_COL_MEMORY_CLOCK;
    case C_TEMP: return PM_COL_TEMPERATURE;
    case C_PLIMIT: return PM_COL_POWER_LIMIT;
    case C_ENF: return PM_COL_ENFORCED_LIMIT;
    case C_PSTATE: return PM_COL_PSTATE;
    default: return 0u;
  }
}

__device__ __forceinline__ double col_value(const pm_trials& T, int c, int64_t i) {
  switch (c) {
    case C_POWER: return col_at(T.power_w, PM_COL_POWER_W, T, i);
    case C_GFX: return col_at(T.graphics_clock_mhz, PM_COL_GRAPHICS_CLOCK, T, i);
    case C_SM: return col_at(T.sm_clock_mhz, PM_COL_SM_CLOCK, T, i);
    case C_MEM: return col_at(T.memory_clock_mhz, PM_COL_MEMORY_CLOCK, T, i);
    case C_TEMP: return col_at(T.temperature_c, PM_COL_TEMPERATURE, T, i);
    case C_PLIMIT: return col_at(T.power_limit_w, PM_COL_POWER_LIMIT, T, i);
    case C_ENF: return col_at(T.enforced_power_limit_w, PM_COL_ENFORCED_LIMIT, T, i);
    default: return col_at(T.pstate, PM_COL_PSTATE, T, i);
  }
}

// ---------------------------------------------------------------------------
// _measure_epochs for one arm (single thread).
__device__ __noinline__ void measure_epochs(const pm_trials& T, const pm_policy& P, int trial, int arm,
                               double phase_start, double phase_end, double whole_ops, double whole_bytes,
                               EpochResult& r, int16_t* order) {
  r.n_inner = 0; r.issue = -1; r.start_s = r.end_s = dnan();
  r.ops = r.bytes = r.slots = dnan(); r.exact = 0;
  const int status = ro(T.epoch_status + (trial * 2 + arm));
  if (status == PM_EP_NONE || status == PM_EP_INVALID_LIST) return;
  if (none(phase_start) || none(phase_end)) { r.issue = 0; return; }
  const int32_t b = ro(T.epoch_offsets + (trial * 2 + arm)), e = ro(T.epoch_offsets + (trial * 2 + arm + 1));
  const int n = e - b;
  if (n < 0 || n > kMaxEpochs) { r.issue = 5; return; }   // the host entry points reject these lists first
  for (int k = 0; k < n; ++k) {
    const double a = ro(T.epoch_start_s + (b + k)), z = ro(T.epoch_end_s + (b + k));
    if (none(a) || none(z) || z <= a || a < phase_start - 1e-6 || z > phase_end + 1e-6) { r.issue = 1; return; }
    const double ops = ro(T.epoch_operations + (b + k));
    if (none(ops) || ops < 0) { r.issue = 2; return; }
    const double bytes = ro(T.epoch_logical_bytes + (b + k));
    if (none(bytes) || bytes < 0) { r.issue = 3; return; }
  }
  if (status == PM_EP_NON_DICT_AFTER) { r.issue = 8; return; }
  // Stable insertion sort by start (Python's list.sort is stable).
  for (int k = 0; k < n; ++k) {
    const double key = ro(T.epoch_start_s + (b + k));
    int j = k - 1;
    while (j >= 0 && ro(T.epoch_start_s + (b + order[j])) > key) { order[j + 1] = order[j]; --j; }
    order[j + 1] = (int16_t)k;
  }
  for (int k = 1; k < n; ++k)
    if (ro(T.epoch_start_s + (b + order[k])) < ro(T.epoch_end_s + (b + order[k - 1])) - 1e-6) { r.issue = 4; return; }
  int first = -1, last = -1, kept = 0;
  for (int k = 0; k < n; ++k) {
    const int i = b + order[k];
    if (ro(T.epoch_start_s + (i)) >= phase_start + P.trim_s - 1e-6 && ro(T.epoch_end_s + (i)) <= phase_end - P.trim_s + 1e-6) {
      if (first < 0) first = k;
      last = k; ++kept;
    }
  }
  if (kept == 0 || ro(T.epoch_end_s + (b + order[last])) - ro(T.epoch_start_s + (b + order[first])) < P.min_measure_s - 1e-6) {
    r.issue = 5; return;
  }
  NeumaierSum so, sb;
  for (int k = 0; k < n; ++k) { so.add(ro(T.epoch_operations + (b + order[k]))); sb.add(ro(T.epoch_logical_bytes + (b + order[k]))); }
  const double counted_ops = so.result(), counted_bytes = sb.result();
  if (!none(whole_ops) && fabs(counted_ops - whole_ops) > fmax(fabs(whole_ops) * 1e-6, 1.0)) { r.issue = 6; return; }
  if (!none(whole_bytes) && fabs(counted_bytes - whole_bytes) > fmax(fabs(whole_bytes) * 1e-6, 1.0)) { r.issue = 7; return; }
  // Inner epochs keep sorted order; they need not be contiguous in it.
  NeumaierSum io, ib, is;
  bool exact = true, slots_ok = true;
  double s0 = dnan(), s1 = dnan();
  int m = 0;
  for (int k = 0; k < n; ++k) {
    const int i = b + order[k];
    if (!(ro(T.epoch_start_s + (i)) >= phase_start + P.trim_s - 1e-6 && ro(T.epoch_end_s + (i)) <= phase_end - P.trim_s + 1e-6)) continue;
    if (m == 0) s0 = ro(T.epoch_start_s + (i));
    s1 = ro(T.epoch_end_s + (i));
    io.add(ro(T.epoch_operations + (i))); ib.add(ro(T.epoch_logical_bytes + (i)));
    const double sl = ro(T.epoch_loop_slots + (i));
    if (none(sl)) slots_ok = false; else is.add(sl);
    exact = exact && ro(T.epoch_counts_exact + (i)) != 0;
    order[m++] = order[k];   // compact kept indices in place (m <= k)
  }
  r.n_inner = m; r.start_s = s0; r.end_s = s1;
  r.ops = io.result(); r.bytes = ib.result();
  r.slots = slots_ok ? is.result() : dnan();
  r.exact = exact ? 1 : 0;
}

// ---------------------------------------------------------------------------
// _phase_stats for slot (trial, p) on window [start, end] after `trim`.
// Writes Shared::po[p] / pf[p].  All threads call it.
// The phase tile lives in dynamic shared memory unless it is too large, then
// in global scratch.  Each case is its own instantiation, so the shared one
// addresses the tile with shared-memory loads and stores.
extern __shared__ double dyn_tile[];
// Radix-select bins of each warp (one copy per CTA for both tile placements).
__shared__ __align__(8) uint32_t g_sel_hist[kThreads / 32][256];

template <bool kSharedTile>
__device__ __noinline__ void phase_stats_impl(const pm_trials& T, const pm_policy& P, Shared& S, double* gtile, int SP,
                                              int trial, int p, double start, double end, double trim, bool idle,
                                              bool aligned) {
  double* sortbuf = kSharedTile ? dyn_tile : gtile;
  double* po = S.po[p];
  const int slot = trial * PM_PHASES + p;
  const int64_t seg_b = T.phase_offsets[slot], seg_e = T.phase_offsets[slot + 1];
  if (threadIdx.x == 0) {
    for (int f = 0; f < PM_PO_COUNT; ++f) po[f] = dnan();
    S.pf[p] = aligned ? (1u << PM_PF_ALIGNED) : 0u;
  }
  __syncthreads();
  if (!T.phase_present[slot]) {
    if (threadIdx.x == 0) S.pf[p] |= 1u << PM_PF_MISSING;
    __syncthreads();
    return;
  }
  if (none(start) || none(end) || end <= start || end - start <= trim * 2) {
    if (threadIdx.x == 0) S.pf[p] |= 1u << PM_PF_INVALID_WINDOW;
    __syncthreads();
    return;
  }
  start = start + trim; end = end - trim;
  const double duration = end - start;
  const double* t = T.t_s;
  // Selected window [lower_bound(start), upper_bound(end)): warp 0 and warp 1
  // search at once, 32 probes per round.
  if (threadIdx.x < 64) {
    const int lane = threadIdx.x & 31;
    const bool upper = threadIdx.x >= 32;
    const int64_t r = warp_bound(t, seg_b, seg_e, upper ? end : start, upper, lane);
    if (lane == 0) {
      if (upper) { S.sel_hi = r; S.cov_hi = r < seg_e ? r + 1 : r; }
      else { S.sel_lo = r; S.cov_lo = r > seg_b ? r - 1 : r; }
    }
  }
  if (threadIdx.x == 64) {
    S.nchange = 0;
    S.distinct_power = -1;
    for (int c = 0; c < C_COUNT; ++c) S.nfin[c] = 0;
  }
  __syncthreads();
  const int64_t lo = S.sel_lo, hi = S.sel_hi, cb = S.cov_lo, ce = S.cov_hi;
  const int nsel = (int)(hi - lo), ncov = (int)(ce - cb);
  // ---- columns to sort: +inf marks "not a value" so finite values lead.
  const double inf = dinf();
  for (int q = threadIdx.x; q < SP; q += blockDim.x) {
    double* col = sortbuf;
    // every load of the sample first, then the stores
    const bool gap = q < ncov - 1, selected = q < nsel;
    const double ta = gap ? ro(t + cb + q) : 0.0, tb = gap ? ro(t + cb + q + 1) : 0.0;
    double v[C_COUNT];
#pragma unroll
    for (int c = C_POWER; c < C_COUNT; ++c) {
      v[c] = inf;
      if (selected && !(T.broadcast_columns & column_bit(c))) v[c] = col_value(T, c, lo + q);
    }
    col[C_GAP * SP + q] = gap ? tb - ta : inf;
    col[C_CHANGE * SP + q] = inf;
#pragma unroll
    for (int c = C_POWER; c < C_COUNT; ++c) {
      if (T.broadcast_columns & column_bit(c)) continue;   // one value for every sample: see the reductions
      col[c * SP + q] = none(v[c]) ? inf : v[c];
    }
  }
  __syncthreads();
  // ---- change instants: selected pairs whose _finite(power) differ.
  // The list is ordered; compact with a CTA prefix count.
  {
    __shared__ int warp_counts[kThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int base = 0;
    for (int q0 = 0; q0 < nsel - 1; q0 += blockDim.x) {
      const int q = q0 + threadIdx.x;
      bool change = false;
      if (q < nsel - 1) {
        const double a = col_at(T.power_w, PM_COL_POWER_W, T, lo + q), b = col_at(T.power_w, PM_COL_POWER_W, T, lo + q + 1);
        change = none(a) != none(b) || (!none(a) && a != b);
      }
      const unsigned ballot = __ballot_sync(0xffffffffu, change);
      if (lane == 0) warp_counts[warp] = __popc(ballot);
      __syncthreads();
      int before = base;
      for (int w = 0; w < warp; ++w) before += warp_counts[w];
      int total = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total += warp_counts[w];
      if (change) {
        const int pos = before + __popc(ballot & ((1u << lane) - 1u));
        // store the change instant temporarily in the CHANGE column
        sortbuf[C_CHANGE * SP + pos] = ro(t + lo + q + 1);
      }
      base += total;
      __syncthreads();
    }
    if (threadIdx.x == 0) S.nchange = base;
    __syncthreads();
    // Gaps between consecutive change instants, in place: each chunk of
    // blockDim.x slots reads its two neighbours before any slot is rewritten.
    const int nch = S.nchange;
    double* ch = sortbuf + C_CHANGE * SP;
    for (int q0 = 0; q0 < SP; q0 += blockDim.x) {
      const int q = q0 + threadIdx.x;
      double g = inf;
      if (q + 1 < nch) g = ch[q + 1] - ch[q];
      __syncthreads();
      if (q < SP) ch[q] = g;
      __syncthreads();
    }
  }
  // The covering samples' times and powers (the energy inputs) are staged
  // by the pass below; the energy counter and the trapezoid terms follow the
  // sort, whose exchange buffers share their columns.
  double* st_t = sortbuf + (size_t)(C_COUNT + S_T) * SP;
  double* st_p = sortbuf + (size_t)(C_COUNT + S_POWER) * SP;
  double* st_m = sortbuf + (size_t)(C_COUNT + S_MEMORY) * SP;
  double* st_r = sortbuf + (size_t)(C_COUNT + S_REL) * SP;
  double* term_p = sortbuf + (size_t)(C_COUNT + S_TERM_P) * SP;
  double* term_m = sortbuf + (size_t)(C_COUNT + S_TERM_M) * SP;
  unsigned long long* pset = reinterpret_cast<unsigned long long*>(sortbuf + (size_t)(C_COUNT + S_SET0) * SP);
  // ---- reductions over the selected samples.
  // Each staged column (finite values, +inf for None) is reduced by one warp:
  // finite count, minimum and maximum.  The flags of the staged clock,
  // temperature, limit and pstate columns follow from those; sample flags,
  // throttle reasons and memory-power sources are read in one pass over the
  // covering samples, which also stages the energy inputs.
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int span = ncov > nsel ? ncov : nsel;          // every staged entry lies below it
    for (int c = warp; c < C_COUNT; c += nwarps) {
      double mn = inf, mx = -inf; int f = 0;
      if (T.broadcast_columns & column_bit(c)) {
        // every selected sample holds the one value: as if staged nsel times
        const double v = col_value(T, c, 0);
        if (!none(v) && nsel > 0) { mn = mx = v; f = nsel; }
      } else {
        const double* col = sortbuf + (size_t)c * SP;
        for (int q = lane; q < span; q += 32) {
          const double v = col[q];
          if (v != inf) { ++f; mn = fmin(mn, v); mx = fmax(mx, v); }
        }
        for (int o = 16; o; o >>= 1) {
          mn = fmin(mn, __shfl_xor_sync(0xffffffffu, mn, o));
          mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          f += __shfl_xor_sync(0xffffffffu, f, o);
        }
      }
      if (lane == 0) { S.cmin[c] = mn; S.cmax[c] = mx; S.nfin[c] = f; }
    }
    uint32_t flags = 0, thr_lo = 0, thr_hi = 0, src_mask = 0, anchor_q = 0x7fffffffu;
    bool neg_power = false;
    for (int q = threadIdx.x; q < ncov; q += blockDim.x) {
      const int64_t i = cb + q;
      const double pw = col_at(T.power_w, PM_COL_POWER_W, T, i);
      const uint16_t sf = col_at(T.sample_flags, PM_COL_SAMPLE_FLAGS, T, i);
      const double mp = col_at(T.memory_power_w, PM_COL_MEMORY_POWER_W, T, i);
      st_t[q] = ro(t + i); st_p[q] = pw; st_m[q] = mp;
      if ((sf & PM_S_ENERGY_ANCHOR) && (uint32_t)q < anchor_q) anchor_q = (uint32_t)q;
      if (!none(pw) && pw < 0) neg_power = true;   // negative power is checked over the covering samples
      if (i < lo || i >= hi) continue;             // the rest concerns the selected samples
      if (!(sf & PM_S_THROTTLE_VALID)) flags |= 1u << PM_PF_THROTTLE_MISSING;
      else {
        const unsigned long long thr = (unsigned long long)col_at(T.throttle_reasons, PM_COL_THROTTLE, T, i) & ~3ull;
        thr_lo |= (uint32_t)thr; thr_hi |= (uint32_t)(thr >> 32);
      }
      if (sf & PM_S_FOREIGN_PID) flags |= 1u << PM_PF_FOREIGN_PID;
      if (sf & PM_S_NO_COMPUTE_INV) flags |= 1u << PM_PF_NO_COMPUTE_INV;
      if (sf & PM_S_NO_GRAPHICS_INV) flags |= 1u << PM_PF_NO_GRAPHICS_INV;
      if (sf & PM_S_MPS) flags |= 1u << PM_PF_MPS;
      if (sf & PM_S_PID_UNKNOWN) flags |= 1u << PM_PF_PID_UNKNOWN;
      if (sf & PM_S_REF_FOREIGN) flags |= 1u << PM_PF_REF_FOREIGN;
      if (sf & PM_S_MEMORY_POWER_SET) {
        const uint8_t src = col_at(T.memory_power_source, PM_COL_MEMORY_SOURCE, T, i);
        if (src) src_mask |= 1u << (src & 15);
      }
    }
    flags = __reduce_or_sync(0xffffffffu, flags);
    anchor_q = __reduce_min_sync(0xffffffffu, anchor_q);
    thr_lo = __reduce_or_sync(0xffffffffu, thr_lo);
    thr_hi = __reduce_or_sync(0xffffffffu, thr_hi);
    src_mask = __reduce_or_sync(0xffffffffu, src_mask);
    const bool any_neg = __any_sync(0xffffffffu, neg_power);
    __shared__ uint32_t red_flags, red_thr_lo, red_thr_hi, red_src;
    __shared__ int red_neg;
    if (threadIdx.x == 0) { red_flags = 0; red_thr_lo = red_thr_hi = 0; red_src = 0; red_neg = 0; S.anchor_q = 0x7fffffff; }
    // the distinct-power set starts empty
    for (int q = threadIdx.x; q < 2 * SP; q += blockDim.x) pset[q] = kSetEmpty;
    __syncthreads();
    if (lane == 0) {
      if (anchor_q != 0x7fffffffu) atomicMin(&S.anchor_q, (int)anchor_q);
      if (flags) atomicOr(&red_flags, flags);
      if (thr_lo) atomicOr(&red_thr_lo, thr_lo);
      if (thr_hi) atomicOr(&red_thr_hi, thr_hi);
      if (src_mask) atomicOr(&red_src, src_mask);
      if (any_neg) red_neg = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t fl = red_flags;
      const unsigned long long thr = ((unsigned long long)red_thr_hi << 32) | red_thr_lo;
      if (S.nfin[C_SM] > 0) fl |= 1u << PM_PF_ANY_SM_FINITE;
      if (S.nfin[C_TEMP] < nsel) fl |= 1u << PM_PF_TEMP_MISSING;
      // "None or <= 0" for some selected sample: a None, or a minimum <= 0
      if (S.nfin[C_GFX] < nsel || S.cmin[C_GFX] <= 0) fl |= 1u << PM_PF_GFX_NONPOS;
      if (S.nfin[C_MEM] < nsel || S.cmin[C_MEM] <= 0) fl |= 1u << PM_PF_MEM_NONPOS;
      if (S.nfin[C_SM] < nsel || S.cmin[C_SM] <= 0) fl |= 1u << PM_PF_SM_NONPOS;
      if (thr) fl |= 1u << PM_PF_THROTTLE_ACTIVE;
      if (red_neg) fl |= 1u << PM_PF_NEGATIVE_POWER;
      S.pf[p] |= fl | (1u << PM_PF_COMPUTED);
      po[PM_PO_THROTTLE_OR] = (double)thr;
      po[PM_PO_MEM_SOURCES] = (double)red_src;
      po[PM_PO_PLIMIT_NONE] = nsel - S.nfin[C_PLIMIT];
      po[PM_PO_ENF_NONE] = nsel - S.nfin[C_ENF];
      po[PM_PO_PSTATE_NONE] = nsel - S.nfin[C_PSTATE];
      // Only columns holding more than one distinct value need a selection;
      // of the power column only its distinct count is used.
      int nm = 0;
      for (int c = 0; c < C_COUNT; ++c)
        if (c != C_POWER && S.nfin[c] > 1 && S.cmin[c] != S.cmax[c]) S.med_cols[nm++] = c;
      S.nmed = nm;
      S.distinct_power = S.nfin[C_POWER] > 1 && S.cmin[C_POWER] != S.cmax[C_POWER] ? 0 : -1;
    }
  }
  __syncthreads();
  // ---- energies: stage the energy counter relative to its anchor while
  // warps 0-2 find the window's edges in the staged times; form the
  // trapezoid terms in parallel; the sums follow, beside the medians.
  __shared__ int s_edge[3];   // upper_bound(start), lower_bound(start), lower_bound(end) over st_t
  __shared__ int s_gap;
  if (threadIdx.x < 96) {
    const int w = threadIdx.x >> 5;
    const int64_t r = warp_bound(st_t, 0, ncov, w == 2 ? end : start, w == 0, threadIdx.x & 31);
    if ((threadIdx.x & 31) == 0) s_edge[w] = (int)r;
  }
  if (threadIdx.x == 0) s_gap = 0;
  {
    const int aq = S.anchor_q;
    const int64_t anchor = aq == 0x7fffffff ? 0 : col_at(T.energy_int, PM_COL_ENERGY_INT, T, cb + aq);
    for (int q = threadIdx.x; q < ncov; q += blockDim.x) {
      const uint16_t sf = col_at(T.sample_flags, PM_COL_SAMPLE_FLAGS, T, cb + q);
      double v;
      if (sf & PM_S_ENERGY_INT) v = (double)(long long)((unsigned long long)col_at(T.energy_int, PM_COL_ENERGY_INT, T, cb + q) - (unsigned long long)anchor);
      else if (sf & PM_S_ENERGY_FLOAT) v = col_at(T.energy_float, PM_COL_ENERGY_FLOAT, T, cb + q) - (double)anchor;
      else v = dnan();
      st_r[q] = isfinite(v) ? v : dnan();
    }
  }
  __syncthreads();
  // Interior samples are covering indices [ia, ib): start < t < end.
  const int ia = s_edge[0], lb_start = s_edge[1], ib = s_edge[2];
  const int nterms = ib > ia ? ib - ia + 1 : 1;
  // _interpolate at x, given i = lower_bound(st_t, x).
  auto value_at = [&](const double* v, double x, int i) -> double {
    if (ncov <= 0 || x < st_t[0] || x > st_t[ncov - 1]) return dnan();
    if (st_t[i] == x) return v[i];
    const double a = v[i - 1], b = v[i];
    if (none(a) || none(b)) return dnan();
    const double ratio = (x - st_t[i - 1]) / (st_t[i] - st_t[i - 1]);
    return a + ratio * (b - a);
  };
  const double p0 = value_at(st_p, start, lb_start), p1 = value_at(st_p, end, ib);
  const double m0 = value_at(st_m, start, lb_start), m1 = value_at(st_m, end, ib);
  bool gap_p = false, gap_m = false;
  for (int k = threadIdx.x; k < nterms; k += blockDim.x) {
    // term k joins point k-1 and point k of [start, interior..., end]
    const double ta = k == 0 ? start : st_t[ia + k - 1];
    const double tb = k == nterms - 1 ? end : st_t[ia + k];
    const double pa = k == 0 ? p0 : st_p[ia + k - 1], pb = k == nterms - 1 ? p1 : st_p[ia + k];
    const double ma = k == 0 ? m0 : st_m[ia + k - 1], mb = k == nterms - 1 ? m1 : st_m[ia + k];
    if (k < nterms - 1) { gap_p |= none(st_p[ia + k]); gap_m |= none(st_m[ia + k]); }
    term_p[k] = (tb - ta) * (pa + pb) * 0.5;
    term_m[k] = (tb - ta) * (ma + mb) * 0.5;
  }
  {
    const unsigned gp = __ballot_sync(0xffffffffu, gap_p), gm = __ballot_sync(0xffffffffu, gap_m);
    if ((threadIdx.x & 31) == 0 && (gp | gm)) atomicOr(&s_gap, (gp ? 1 : 0) | (gm ? 2 : 0));
  }
  __syncthreads();
  gap_p = (s_gap & 1) != 0;
  gap_m = (s_gap & 2) != 0;
  // ---- side by side, all independent of one another: each energy sum on
  // one lane (lane 0 of the last three warps) in the reference's order; the
  // median of each varying column by one warp from warp 0 (warp_median: a
  // median needs order statistics (n-1)/2 and n/2 only); the distinct
  // finite powers into a hash set by the warps from the first one without a
  // column (at most the last three).
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    if (lane == 0 && warp == nwarps - 1) {
      double energy = dnan();
      if (!none(p0) && !none(p1) && end > start && !gap_p) energy = neumaier_sum(term_p, nterms);
      po[PM_PO_ENERGY_J] = energy;
      po[PM_PO_INTEGRATED_POWER_W] = none(energy) ? dnan() : energy / duration;
    } else if (lane == 0 && warp == nwarps - 2) {
      double me = dnan();
      if (!none(m0) && !none(m1) && end > start && !gap_m) me = neumaier_sum(term_m, nterms);
      po[PM_PO_MEMORY_ENERGY_J] = me;
      po[PM_PO_MEMORY_POWER_W] = none(me) ? dnan() : me / duration;
    } else if (lane == 0 && warp == nwarps - 3) {
      const double c0 = value_at(st_r, start, lb_start), c1 = value_at(st_r, end, ib);
      bool reset = false, have = false;
      double prev = 0.0;
      for (int q = 0; q < ncov; ++q) {
        const double v = st_r[q];
        if (none(v)) continue;
        if (have && v < prev) reset = true;
        prev = v; have = true;
      }
      double counter = dnan();
      if (!none(c0) && !none(c1)) {
        if (reset || c1 < c0) atomicOr(&S.pf[p], 1u << PM_PF_COUNTER_RESET);
        else counter = (c1 - c0) / 1000.0;
      }
      po[PM_PO_COUNTER_J] = counter;
    }
    const int span = ncov > nsel ? ncov : nsel;
    const int nmed = S.nmed;
    for (int a = warp; a < nmed; a += nwarps) {
      const int c = S.med_cols[a];
      const double m = warp_median(sortbuf + (size_t)c * SP, span, S.nfin[c], S.cmin[c], S.cmax[c], g_sel_hist[warp]);
      if (lane == 0) S.cmed[c] = m;
    }
    if (S.distinct_power >= 0) {
      const int first = nmed < nwarps - 3 ? nmed : nwarps - 3;
      if (warp >= first) {
        const double* pw = sortbuf + (size_t)C_POWER * SP;
        int added = 0;
        for (int q = threadIdx.x - first * 32; q < nsel; q += (nwarps - first) * 32)
          if (pw[q] != inf) added += set_insert(pset, 2 * SP, pw[q]);
        added = __reduce_add_sync(0xffffffffu, added);
        if (lane == 0 && added) atomicAdd(&S.distinct_power, added);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    po[PM_PO_START_S] = start; po[PM_PO_END_S] = end; po[PM_PO_DURATION_S] = duration;
    po[PM_PO_MIDPOINT_S] = (start + end) / 2;
    po[PM_PO_SAMPLES] = nsel;
    po[PM_PO_SEL_LO] = (double)(lo - seg_b); po[PM_PO_SEL_HI] = (double)(hi - seg_b);
    po[PM_PO_COV_LO] = (double)(cb - seg_b); po[PM_PO_COV_HI] = (double)(ce - seg_b);
    // A column that was not sorted holds one repeated value: its median,
    // minimum and maximum are that value.
    auto column_median = [&](int c) -> double {
      const int n = S.nfin[c];
      if (n == 0) return dnan();
      if (S.cmin[c] == S.cmax[c]) return S.cmin[c];
      return S.cmed[c];
    };
    const int ngap = S.nfin[C_GAP];
    po[PM_PO_GAP_MEDIAN_S] = column_median(C_GAP);
    po[PM_PO_GAP_MAX_S] = ngap ? S.cmax[C_GAP] : dnan();
    po[PM_PO_CHANGE_MEDIAN_S] = column_median(C_CHANGE);
    {
      // A varying power column's distinct values were counted in a hash
      // set; otherwise the column holds one repeated value or none.
      const int n = S.nfin[C_POWER];
      po[PM_PO_DISTINCT_POWER] = S.distinct_power >= 0 ? S.distinct_power : (n ? 1 : 0);
    }
    const int stat_cols[7] = {C_GFX, C_SM, C_MEM, C_TEMP, C_PLIMIT, C_ENF, C_PSTATE};
    const int med_slot[7] = {PM_PO_GFX_MED, PM_PO_SM_MED, PM_PO_MEM_MED, PM_PO_TEMP_MED, PM_PO_PLIMIT_MED, PM_PO_ENF_MED, PM_PO_PSTATE_MED};
    const int min_slot[7] = {PM_PO_GFX_MIN, PM_PO_SM_MIN, PM_PO_MEM_MIN, PM_PO_TEMP_MIN, PM_PO_PLIMIT_MIN, PM_PO_ENF_MIN, PM_PO_PSTATE_MIN};
    const int max_slot[7] = {PM_PO_GFX_MAX, PM_PO_SM_MAX, PM_PO_MEM_MAX, PM_PO_TEMP_MAX, PM_PO_PLIMIT_MAX, PM_PO_ENF_MAX, PM_PO_PSTATE_MAX};
    for (int k = 0; k < 7; ++k) {
      const int c = stat_cols[k], n = S.nfin[c];
      po[med_slot[k]] = column_median(c);
      po[min_slot[k]] = n ? S.cmin[c] : dnan();
      po[max_slot[k]] = n ? S.cmax[c] : dnan();
    }
    po[PM_PO_PLIMIT_FIN] = S.nfin[C_PLIMIT]; po[PM_PO_ENF_FIN] = S.nfin[C_ENF]; po[PM_PO_PSTATE_FIN] = S.nfin[C_PSTATE];
    // power_w: counter rate if present else trapezoid rate
    const double energy = po[PM_PO_ENERGY_J], counter = po[PM_PO_COUNTER_J];
    po[PM_PO_POWER_W] = !none(counter) ? counter / duration : po[PM_PO_INTEGRATED_POWER_W];
    uint32_t f = S.pf[p];
    const double minimum = idle ? P.min_idle_s : P.min_measure_s;
    if (duration + 1e-9 < minimum) f |= 1u << PM_PF_SHORT_PLATEAU;
    if (nsel < P.min_samples) f |= 1u << PM_PF_TOO_FEW_SAMPLES;
    if (ngap && S.cmax[C_GAP] > P.max_sample_gap_s) f |= 1u << PM_PF_TELEMETRY_GAP;
    if (none(energy)) f |= 1u << PM_PF_MISSING_POWER_COVERAGE;
    if (!none(counter) && !none(energy) && energy > 0) {
      const double d = fabs(counter - energy) / energy;
      po[PM_PO_DISAGREEMENT] = d;
      if (d > P.counter_disagreement_fraction) f |= 1u << PM_PF_COUNTER_DISAGREEMENT;
    }
    S.pf[p] = f;
  }
  __syncthreads();
}

// _phase_stats on the tile in global scratch (gtile != NULL) or in shared memory.
__device__ __forceinline__ void phase_stats(const pm_trials& T, const pm_policy& P, Shared& S, double* gtile, int SP,
                                            int trial, int p, double start, double end, double trim, bool idle,
                                            bool aligned) {
  if (gtile) phase_stats_impl<false>(T, P, S, gtile, SP, trial, p, start, end, trim, idle, aligned);
  else phase_stats_impl<true>(T, P, S, gtile, SP, trial, p, start, end, trim, idle, aligned);
}

__device__ __forceinline__ double fin(double x) { return x; }   // NaN already means None
__device__ __forceinline__ bool truthy(double x) { return !none(x) && x != 0.0; }

// _idle_at(pre, post, active, field) on phase outputs.
__device__ double idle_at(const double* pre, const double* post, const double* act, int field) {
  const double a = pre[field], b = post[field];
  const double t0 = pre[PM_PO_MIDPOINT_S], t1 = post[PM_PO_MIDPOINT_S], t = act[PM_PO_MIDPOINT_S];
  if (none(a) || none(b) || none(t0) || none(t1) || none(t) || t1 <= t0 || !(t0 <= t && t <= t1)) return dnan();
  return a + (b - a) * (t - t0) / (t1 - t0);
}

// Deliver one trial's metric row and valid flag to every rank's gathered
// buffers (peer stores over NVLink); the last CTA of the launch to get here
// raises this rank's arrival flag on every rank.  Each CTA counts with an
// acquire-release add (GPU scope: every counting CTA is on this GPU), so its
// row stores are released to the counter; the last CTA, having acquired every
// earlier count, releases them all with its system-scope flag stores: a rank
// that acquires the flag sees all of this launch's rows.
__device__ __noinline__ void deliver_rows(const pm_peer_rows& X, int trial, const double* m, uint8_t valid,
                                          uint32_t n_trials) {
  const size_t row = (size_t)(X.row_offset + trial);
  for (int r = 0; r < X.n_ranks; ++r) {
    double* dst = X.metrics[r] + row * PM_N_METRICS;
    for (int k = 0; k < PM_N_METRICS; ++k) dst[k] = m[k];
    X.valid[r][row] = valid;
  }
  uint32_t prev;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(X.done) : "memory");
  if (prev + 1u == X.epoch * n_trials)
    for (int r = 0; r < X.n_ranks; ++r)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(X.flags[r] + X.rank), "r"(X.epoch) : "memory");
}

__global__ void __launch_bounds__(kThreads)
analyze_kernel(pm_trials T, pm_policy P, pm_trial_results R, int SP, double* gscratch, pm_peer_rows X) {
  __shared__ Shared S;
  const int trial = blockIdx.x;
  double* sortbuf = gscratch ? gscratch + (size_t)blockIdx.x * kTileColumns * SP : nullptr;   // NULL: shared tile
  // The trial's scalars, read many times by the trial-level code: one coalesced load.
  __shared__ double s_ts[PM_TS_COUNT];
  __shared__ uint32_t s_scan;   // per-sample state scans: one bit per check failed
  for (int i = threadIdx.x; i < PM_TS_COUNT; i += blockDim.x) s_ts[i] = T.trial_scalars[(size_t)trial * PM_TS_COUNT + i];
  if (threadIdx.x == 0) s_scan = 0;
  __syncthreads();
  const double* ts = s_ts;
  const uint32_t tflags = T.trial_flags[trial];
  const int wl = tflags & PM_T_WORKLOAD_MASK;
  const bool tensor = wl == PM_WL_TENSOR, memory = wl == PM_WL_MEMORY, sfu = wl == PM_WL_SFU, nonlinear = wl == PM_WL_NONLINEAR;
  const bool energy_wl = wl != PM_WL_OTHER;
  const int ms = trial * PM_PHASES;

  // The two arms' epochs are independent: one thread of warp 0 and one of warp 1.
  if (threadIdx.x == 0) {
    measure_epochs(T, P, trial, 0, T.phase_present[ms + PM_MEASURE] ? T.phase_start_s[ms + PM_MEASURE] : dnan(),
                   T.phase_present[ms + PM_MEASURE] ? T.phase_end_s[ms + PM_MEASURE] : dnan(),
                   ts[PM_TS_BENCH_OPERATIONS], ts[PM_TS_BENCH_LOGICAL_BYTES], S.ep[0], S.order[0]);
  } else if (threadIdx.x == 32) {
    if (T.phase_present[ms + PM_REFERENCE])
      measure_epochs(T, P, trial, 1, T.phase_start_s[ms + PM_REFERENCE], T.phase_end_s[ms + PM_REFERENCE],
                     ts[PM_TS_REF_OPERATIONS], ts[PM_TS_REF_LOGICAL_BYTES], S.ep[1], S.order[1]);
    else { S.ep[1].n_inner = 0; S.ep[1].issue = -1; S.ep[1].exact = 0; }
  }
  __syncthreads();
  phase_stats(T, P, S, sortbuf, SP, trial, PM_IDLE_PRE, T.phase_start_s[ms + PM_IDLE_PRE], T.phase_end_s[ms + PM_IDLE_PRE], P.idle_trim_s, true, false);
  phase_stats(T, P, S, sortbuf, SP, trial, PM_IDLE_POST, T.phase_start_s[ms + PM_IDLE_POST], T.phase_end_s[ms + PM_IDLE_POST], P.idle_trim_s, true, false);
  if (S.ep[0].n_inner > 0)
    phase_stats(T, P, S, sortbuf, SP, trial, PM_MEASURE, S.ep[0].start_s, S.ep[0].end_s, 0.0, false, true);
  else
    phase_stats(T, P, S, sortbuf, SP, trial, PM_MEASURE, T.phase_start_s[ms + PM_MEASURE], T.phase_end_s[ms + PM_MEASURE], P.trim_s, false, false);
  const bool has_ref = T.phase_present[ms + PM_REFERENCE] != 0;
  if (has_ref) {
    if (S.ep[1].n_inner > 0)
      phase_stats(T, P, S, sortbuf, SP, trial, PM_REFERENCE, S.ep[1].start_s, S.ep[1].end_s, 0.0, false, true);
    else
      phase_stats(T, P, S, sortbuf, SP, trial, PM_REFERENCE, T.phase_start_s[ms + PM_REFERENCE], T.phase_end_s[ms + PM_REFERENCE], P.trim_s, false, false);
  } else if (threadIdx.x == 0) {
    for (int f = 0; f < PM_PO_COUNT; ++f) S.po[PM_REFERENCE][f] = dnan();
    S.pf[PM_REFERENCE] = 1u << PM_PF_MISSING;
  }
  const bool has_control = T.phase_present[ms + PM_CONTROL] != 0;
  if (has_control) {
    phase_stats(T, P, S, sortbuf, SP, trial, PM_CONTROL, T.phase_start_s[ms + PM_CONTROL], T.phase_end_s[ms + PM_CONTROL], P.trim_s, false, false);
  } else if (threadIdx.x == 0) {
    for (int f = 0; f < PM_PO_COUNT; ++f) S.po[PM_CONTROL][f] = dnan();
    S.pf[PM_CONTROL] = 1u << PM_PF_MISSING;
  }
  __syncthreads();
  const double* pre = S.po[PM_IDLE_PRE];
  const double* post = S.po[PM_IDLE_POST];
  const double* mea = S.po[PM_MEASURE];
  const double* ref = S.po[PM_REFERENCE];
  const uint32_t mf = S.pf[PM_MEASURE];

  // ---- per-sample baseline and paired state scans (all threads) -------------
  // analyze_trial:780-805: each idle phase's selected samples vs the active
  // median (clocks relative, temperature absolute); _paired_reference_contrast
  // :335-342: the reference's selected samples vs the treatment median (all
  // absolute).  Every check of a phase is made in one pass over its samples
  // (check k of phase j is bit 4j + k: graphics, memory and SM clock, then
  // temperature); a sample with no value fails a check as well.
  const bool base_sm = ((mf | S.pf[PM_IDLE_PRE] | S.pf[PM_IDLE_POST]) >> PM_PF_ANY_SM_FINITE) & 1u;
  const bool paired_sm = ((mf | S.pf[PM_REFERENCE]) >> PM_PF_ANY_SM_FINITE) & 1u;
  const int clock_cols[3] = {C_GFX, C_MEM, C_SM};
  const int med_slot[3] = {PM_PO_GFX_MED, PM_PO_MEM_MED, PM_PO_SM_MED};
  {
    uint32_t bad = 0;
    const int scan_phase[3] = {PM_IDLE_PRE, PM_IDLE_POST, PM_REFERENCE};
    for (int j = 0; j < 3; ++j) {
      const int ph = scan_phase[j];
      const bool ref = j == 2;
      if (ref && !has_ref) continue;
      bool on[4];
      double center[4], tol[4];
      const int nclk = (ref ? paired_sm : base_sm) ? 3 : 2;
      for (int k = 0; k < 3; ++k) {
        const double active = mea[med_slot[k]];
        if (ref) {
          on[k] = k < nclk;
          center[k] = none(active) ? 0.0 : active;
          tol[k] = center[k] * P.clock_tolerance_fraction;
        } else {
          on[k] = k < nclk && !none(active) && active > 0;
          center[k] = active;
          tol[k] = P.clock_tolerance_fraction;   // relative
        }
      }
      const double at = mea[PM_PO_TEMP_MED];
      on[3] = ref || !none(at);
      center[3] = none(at) ? 0.0 : at;
      tol[3] = P.max_temperature_drift_c;
      if (!(S.pf[ph] & (1u << PM_PF_COMPUTED)) || !(on[0] || on[1] || on[2] || on[3])) continue;
      const int64_t b = T.phase_offsets[trial * PM_PHASES + ph];
      const int64_t lo = b + (int64_t)S.po[ph][PM_PO_SEL_LO], hi = b + (int64_t)S.po[ph][PM_PO_SEL_HI];
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (!on[k]) continue;
          const double v = col_value(T, k < 3 ? clock_cols[k] : C_TEMP, i);
          const double d = fabs(v - center[k]);
          const bool fail = none(v) || ((!ref && k < 3) ? (d / center[k] > tol[k]) : (d > tol[k]));
          if (fail) bad |= 1u << (4 * j + k);
        }
      }
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0 && bad) atomicOr(&s_scan, bad);
    // The phase records are final: all threads write them out, and fill the
    // trial's scalar and metric rows with None (thread 0 sets the rest after
    // the barrier).
    for (int i = threadIdx.x; i < PM_PHASES * PM_PO_COUNT; i += blockDim.x)
      R.phase_out[(size_t)trial * PM_PHASES * PM_PO_COUNT + i] = S.po[i / PM_PO_COUNT][i % PM_PO_COUNT];
    if (threadIdx.x < PM_PHASES) R.phase_flags[trial * PM_PHASES + threadIdx.x] = S.pf[threadIdx.x];
    for (int i = threadIdx.x; i < PM_TO_COUNT; i += blockDim.x) R.trial_out[(size_t)trial * PM_TO_COUNT + i] = dnan();
    for (int i = threadIdx.x; i < PM_N_METRICS; i += blockDim.x) R.metrics[(size_t)trial * PM_N_METRICS + i] = dnan();
    __syncthreads();
  }
  const uint32_t scan = s_scan;
  const bool scan_idle_clock[2] = {(scan & 0x7u) != 0, (scan & 0x70u) != 0};
  const bool scan_idle_temp[2] = {(scan & 0x8u) != 0, (scan & 0x80u) != 0};
  const bool scan_ref[4] = {(scan & 0x100u) != 0, (scan & 0x200u) != 0, (scan & 0x400u) != 0, (scan & 0x800u) != 0};

  if (threadIdx.x != 0) return;
  // ---- trial scalars and gates (thread 0) ----------------------------------
  double* to = R.trial_out + (size_t)trial * PM_TO_COUNT;   // filled with None above
  uint64_t iss = 0, base = 0, pair = 0, warn = 0;
  auto phase_issue_bits = [&](uint32_t f) -> uint64_t {
    uint64_t b = 0;
    if (f & (1u << PM_PF_MISSING)) b |= 1ull << 0;
    if (f & (1u << PM_PF_INVALID_WINDOW)) b |= 1ull << 1;
    if (f & (1u << PM_PF_SHORT_PLATEAU)) b |= 1ull << 2;
    if (f & (1u << PM_PF_TOO_FEW_SAMPLES)) b |= 1ull << 3;
    if (f & (1u << PM_PF_TELEMETRY_GAP)) b |= 1ull << 4;
    if (f & (1u << PM_PF_NEGATIVE_POWER)) b |= 1ull << 5;
    if (f & (1u << PM_PF_MISSING_POWER_COVERAGE)) b |= 1ull << 6;
    if (f & (1u << PM_PF_COUNTER_DISAGREEMENT)) b |= 1ull << 7;
    return b;
  };
  iss |= phase_issue_bits(mf) << PM_IT_M_MISSING_PHASE;
  if (S.ep[0].issue >= 0) iss |= 1ull << (PM_IT_EP_PHASE_WINDOW + S.ep[0].issue);
  base |= phase_issue_bits(S.pf[PM_IDLE_PRE]) << PM_IB_PRE_MISSING_PHASE;
  base |= phase_issue_bits(S.pf[PM_IDLE_POST]) << PM_IB_POST_MISSING_PHASE;
  if (S.pf[PM_IDLE_PRE] & (1u << PM_PF_COUNTER_RESET)) warn |= 1ull << PM_W_COUNTER_RESET_PRE;
  if (mf & (1u << PM_PF_COUNTER_RESET)) warn |= 1ull << PM_W_COUNTER_RESET_MEASURE;
  if (S.pf[PM_IDLE_POST] & (1u << PM_PF_COUNTER_RESET)) warn |= 1ull << PM_W_COUNTER_RESET_POST;
  if (has_control && (S.pf[PM_CONTROL] & (1u << PM_PF_COUNTER_RESET))) warn |= 1ull << PM_W_COUNTER_RESET_CONTROL;

  // Requested vs achieved clocks (analysis.py:631-646).
  const bool treat_sm = (mf >> PM_PF_ANY_SM_FINITE) & 1u;
  const double req[3] = {ts[PM_TS_REQ_GRAPHICS_MHZ], ts[PM_TS_REQ_MEMORY_MHZ], ts[PM_TS_REQ_SM_MHZ]};
  const int min_slot[3] = {PM_PO_GFX_MIN, PM_PO_MEM_MIN, PM_PO_SM_MIN};
  const int max_slot[3] = {PM_PO_GFX_MAX, PM_PO_MEM_MAX, PM_PO_SM_MAX};
  const int nonpos_flag[3] = {PM_PF_GFX_NONPOS, PM_PF_MEM_NONPOS, PM_PF_SM_NONPOS};
  for (int k = 0; k < (treat_sm ? 3 : 2); ++k) {
    const double actual = mea[med_slot[k]];
    if (!none(req[k]) && req[k] > 0) {
      if (none(actual)) iss |= 1ull << (PM_IT_MISSING_CLOCK_GFX + k);
      else if (fabs(actual - req[k]) / req[k] > P.clock_tolerance_fraction) iss |= 1ull << (PM_IT_CLOCK_MISMATCH_GFX + k);
    } else if (k != 2) {
      warn |= 1ull << (PM_W_UNCONTROLLED_GFX + k);
    }
    const double low = mea[min_slot[k]], high = mea[max_slot[k]];
    if (truthy(actual) && !none(low) && !none(high) && (high - low) / actual > P.max_clock_drift_fraction)
      iss |= 1ull << (PM_IT_CLOCK_DRIFT_GFX + k);
  }
  {
    const double lo_t = mea[PM_PO_TEMP_MIN], hi_t = mea[PM_PO_TEMP_MAX];
    if (!none(lo_t) && !none(hi_t) && hi_t - lo_t > P.max_temperature_drift_c) iss |= 1ull << PM_IT_TEMPERATURE_DRIFT;
  }
  const bool sel_any = truthy(mea[PM_PO_SAMPLES]);
  if (sel_any && (mf & (1u << PM_PF_TEMP_MISSING))) iss |= 1ull << PM_IT_MISSING_TEMPERATURE;
  for (int k = 0; k < (treat_sm ? 3 : 2); ++k)
    if (sel_any && (mf & (1u << nonpos_flag[k]))) iss |= 1ull << (PM_IT_MISSING_CLOCK_GFX + k);
  if (sel_any && (mf & (1u << PM_PF_THROTTLE_MISSING))) iss |= 1ull << PM_IT_MISSING_THROTTLING;
  const double thr = none(mea[PM_PO_THROTTLE_OR]) ? 0.0 : mea[PM_PO_THROTTLE_OR];
  if (thr != 0.0) iss |= 1ull << PM_IT_ACTIVE_THROTTLING;
  // Process inventory: measure -> issues, other phases (idle, control) -> baseline.
  if (mf & (1u << PM_PF_NO_COMPUTE_INV)) iss |= 1ull << PM_IT_MISSING_INV_COMPUTE;
  if (mf & (1u << PM_PF_NO_GRAPHICS_INV)) iss |= 1ull << PM_IT_MISSING_INV_GRAPHICS;
  if (mf & (1u << PM_PF_PID_UNKNOWN)) iss |= 1ull << PM_IT_MISSING_MEASUREMENT_PID;
  if (mf & (1u << PM_PF_FOREIGN_PID)) iss |= 1ull << PM_IT_OTHER_GPU_PROCESSES;
  if (mf & (1u << PM_PF_MPS)) iss |= 1ull << PM_IT_MPS_ACTIVE;
  {
    uint32_t of = S.pf[PM_IDLE_PRE] | S.pf[PM_IDLE_POST] | (has_control ? S.pf[PM_CONTROL] : 0u);
    if (of & (1u << PM_PF_NO_COMPUTE_INV)) base |= 1ull << PM_IB_B_MISSING_INV_COMPUTE;
    if (of & (1u << PM_PF_NO_GRAPHICS_INV)) base |= 1ull << PM_IB_B_MISSING_INV_GRAPHICS;
    if (of & (1u << PM_PF_PID_UNKNOWN)) base |= 1ull << PM_IB_B_MISSING_MEASUREMENT_PID;
    if (of & (1u << PM_PF_FOREIGN_PID)) base |= 1ull << PM_IB_B_OTHER_GPU_PROCESSES;
    if (of & (1u << PM_PF_MPS)) base |= 1ull << PM_IB_B_MPS_ACTIVE;
  }
  // Idle delta (analysis.py:713-727).
  const double idle_power = idle_at(pre, post, mea, PM_PO_POWER_W);
  const double idle_memory_power = idle_at(pre, post, mea, PM_PO_MEMORY_POWER_W);
  {
    const double a = pre[PM_PO_POWER_W], b = post[PM_PO_POWER_W];
    if (!none(a) && !none(b)) {
      const double den = fmax((a + b) / 2, 1e-9);
      if (fabs(a - b) / den > P.max_idle_drift_fraction) base |= 1ull << PM_IB_IDLE_DRIFT;
    }
  }
  const double duration = mea[PM_PO_DURATION_S];
  double total = mea[PM_PO_COUNTER_J];
  bool trapezoid = false;
  if (none(total)) { total = mea[PM_PO_ENERGY_J]; trapezoid = true; }
  const double board_power = (!none(total) && truthy(duration) && duration > 0) ? total / duration : dnan();
  const double idle_energy = (!none(idle_power) && truthy(duration)) ? idle_power * duration : dnan();
  const double incremental = (!none(total) && !none(idle_energy)) ? total - idle_energy : dnan();
  if (none(idle_power)) base |= 1ull << PM_IB_MISSING_IDLE;
  if (!none(incremental) && incremental < 0) base |= 1ull << PM_IB_NEGATIVE_INCREMENTAL;
  const double device_duration = ts[PM_TS_BENCH_DURATION_S];
  const double host_duration = ts[PM_TS_BENCH_HOST_DURATION_S];
  const double measured_duration = truthy(host_duration) ? host_duration : device_duration;
  if (truthy(device_duration) && truthy(measured_duration) && fabs(device_duration - measured_duration) / measured_duration > 0.05)
    iss |= 1ull << PM_IT_DURATION_DISAGREEMENT;
  const double operations = ts[PM_TS_BENCH_OPERATIONS], logical_bytes = ts[PM_TS_BENCH_LOGICAL_BYTES];
  const bool md_ok = truthy(measured_duration) && measured_duration > 0;
  double ops_rate = (!none(operations) && md_ok) ? operations / measured_duration : dnan();
  double byte_rate = (!none(logical_bytes) && md_ok) ? logical_bytes / measured_duration : dnan();
  const EpochResult& E = S.ep[0];
  const bool have_epochs = E.n_inner > 0 && E.issue < 0;
  const bool exact = have_epochs && E.exact;
  const double counted_ops = have_epochs ? E.ops : dnan();
  const double counted_bytes = have_epochs ? E.bytes : dnan();
  if (have_epochs && truthy(duration) && duration > 0) { ops_rate = counted_ops / duration; byte_rate = counted_bytes / duration; }
  if (!exact) warn |= 1ull << PM_W_ALIGNMENT_UNVERIFIED;
  if (none(measured_duration) || measured_duration <= 0) iss |= 1ull << PM_IT_MISSING_BENCH_DURATION;
  if (tensor && (none(ops_rate) || ops_rate <= 0)) iss |= 1ull << PM_IT_MISSING_OPERATION_COUNT;
  if (memory && (none(byte_rate) || byte_rate <= 0)) iss |= 1ull << PM_IT_MISSING_LOGICAL_BYTE_COUNT;
  if (nonlinear && !exact) iss |= 1ull << PM_IT_NONLINEAR_EPOCHS;
  if (sfu && !exact) iss |= 1ull << PM_IT_SFU_EPOCHS;
  const double incremental_power = (!none(incremental) && truthy(duration)) ? incremental / duration : dnan();
  const double rail_energy = mea[PM_PO_MEMORY_ENERGY_J];
  double rail_incremental = (!none(rail_energy) && !none(idle_memory_power) && truthy(duration))
                                ? rail_energy - idle_memory_power * duration : dnan();
  {
    unsigned srcs = (unsigned)(none(pre[PM_PO_MEM_SOURCES]) ? 0 : pre[PM_PO_MEM_SOURCES]) |
                    (unsigned)(none(mea[PM_PO_MEM_SOURCES]) ? 0 : mea[PM_PO_MEM_SOURCES]) |
                    (unsigned)(none(post[PM_PO_MEM_SOURCES]) ? 0 : post[PM_PO_MEM_SOURCES]) |
                    (has_control && !none(S.po[PM_CONTROL][PM_PO_MEM_SOURCES]) ? (unsigned)S.po[PM_CONTROL][PM_PO_MEM_SOURCES] : 0u);
    if (__popc(srcs) > 1) { warn |= 1ull << PM_W_RAIL_SOURCE_CHANGED; rail_incremental = dnan(); }
  }
  // power_limit = median(selected) or record-level fallback (analysis.py:781-783)
  double power_limit = mea[PM_PO_PLIMIT_MED];
  if (!truthy(power_limit)) power_limit = ts[PM_TS_POWER_LIMIT_FALLBACK_W];
  double tensor_peak = dnan();
  const bool peak_sm = truthy(mea[PM_PO_SM_MED]) && mea[PM_PO_SM_MED] > 0;
  const double peak_clock = peak_sm ? mea[PM_PO_SM_MED] : mea[PM_PO_GFX_MED];
  if (tensor && !none(peak_clock) && peak_clock > 0) {
    if (tflags & PM_T_TENSOR_PEAK_KNOWN) {
      tensor_peak = ts[PM_TS_TENSOR_FLOPS_PER_CLOCK] * peak_clock * 1e6 / 1e12;
      if (!peak_sm) warn |= 1ull << PM_W_PEAK_GRAPHICS_PROXY;
    } else {
      warn |= 1ull << PM_W_PEAK_UNAVAILABLE;
    }
  }
  // Baseline state matching (analysis.py:801-835).
  bool clock_matched = true, temp_matched = true, cap_matched = true;
  bool enf_compared = false, pst_compared = false, state_mismatch = false;
  const double* idles[2] = {pre, post};
  const int base_ph[2] = {PM_IDLE_PRE, PM_IDLE_POST};
  for (int side = 0; side < 2; ++side) {
    const double* bp = idles[side];
    const int dbase = side ? PM_TO_DPOST_GFX : PM_TO_DPRE_GFX;
    for (int k = 0; k < (base_sm ? 3 : 2); ++k) {
      const double ac = mea[med_slot[k]], ic = bp[med_slot[k]];
      to[dbase + k] = (!none(ac) && !none(ic)) ? ac - ic : dnan();
      if (none(ac) || none(ic) || ac <= 0 || fabs(ac - ic) / ac > P.clock_tolerance_fraction) clock_matched = false;
    }
    if (scan_idle_clock[side]) clock_matched = false;
    const double at = mea[PM_PO_TEMP_MED], it = bp[PM_PO_TEMP_MED];
    to[dbase + 3] = (!none(at) && !none(it)) ? at - it : dnan();
    if (none(at) || none(it) || fabs(at - it) > P.max_temperature_drift_c) temp_matched = false;
    if (scan_idle_temp[side]) temp_matched = false;
    // caps: set equality of _finite(power_limit_w) over selected samples
    {
      const bool a_single = mea[PM_PO_PLIMIT_NONE] == 0 && mea[PM_PO_PLIMIT_FIN] > 0 && mea[PM_PO_PLIMIT_MIN] == mea[PM_PO_PLIMIT_MAX];
      const bool b_single = bp[PM_PO_PLIMIT_NONE] == 0 && bp[PM_PO_PLIMIT_FIN] > 0 && bp[PM_PO_PLIMIT_MIN] == bp[PM_PO_PLIMIT_MAX];
      const bool a_has_none = !(mea[PM_PO_PLIMIT_NONE] == 0) ;
      const bool b_has_none = !(bp[PM_PO_PLIMIT_NONE] == 0);
      if (a_has_none || b_has_none || !a_single || !b_single || mea[PM_PO_PLIMIT_MIN] != bp[PM_PO_PLIMIT_MIN]) cap_matched = false;
    }
    const int fields[2][5] = {{PM_PO_ENF_NONE, PM_PO_ENF_FIN, PM_PO_ENF_MIN, PM_PO_ENF_MAX, PM_PO_ENF_MED},
                              {PM_PO_PSTATE_NONE, PM_PO_PSTATE_FIN, PM_PO_PSTATE_MIN, PM_PO_PSTATE_MAX, PM_PO_PSTATE_MED}};
    for (int g = 0; g < 2; ++g) {
      const int* F = fields[g];
      const double an = none(mea[F[0]]) ? 0 : mea[F[0]], af = none(mea[F[1]]) ? 0 : mea[F[1]];
      const double bn = none(bp[F[0]]) ? 0 : bp[F[0]], bf = none(bp[F[1]]) ? 0 : bp[F[1]];
      if (af + bf > 0) {
        if (g == 0) enf_compared = true; else pst_compared = true;
        const double amed = truthy(mea[F[4]]) ? mea[F[4]] : 0.0, bmed = truthy(bp[F[4]]) ? bp[F[4]] : 0.0;
        to[dbase + 4 + g] = (an == 0 && bn == 0) ? amed - bmed : dnan();
        const bool a_single = an == 0 && af > 0 && mea[F[2]] == mea[F[3]];
        const bool b_single = bn == 0 && bf > 0 && bp[F[2]] == bp[F[3]];
        if (an > 0 || bn > 0 || !a_single || !b_single || mea[F[2]] != bp[F[2]]) {
          base |= 1ull << (side ? (g ? PM_IB_STATE_POST_PSTATE : PM_IB_STATE_POST_ENF) : (g ? PM_IB_STATE_PRE_PSTATE : PM_IB_STATE_PRE_ENF));
          state_mismatch = true;
        }
      }
    }
    (void)base_ph;
  }
  if (state_mismatch) warn |= 1ull << PM_W_STATE_MISMATCH;
  if (!cap_matched) warn |= 1ull << PM_W_CAP_MISMATCH;
  if (!clock_matched) warn |= 1ull << PM_W_CLOCK_MISMATCH;
  if (!temp_matched) warn |= 1ull << PM_W_TEMP_MISMATCH;

  const bool host_issues = tflags & PM_T_HOST_ISSUES;
  const bool valid = !host_issues && iss == 0;
  const bool baseline_valid = !(tflags & PM_T_HOST_BASELINE) && base == 0;
  const bool idle_inc_eligible = valid && baseline_valid && exact && clock_matched && temp_matched && cap_matched;

  to[PM_TO_DURATION_S] = duration;
  to[PM_TO_BENCH_MEASURED_DURATION_S] = measured_duration;
  to[PM_TO_BENCH_DEVICE_DURATION_S] = device_duration;
  to[PM_TO_IDLE_POWER_W] = idle_power; to[PM_TO_IDLE_MEMORY_POWER_W] = idle_memory_power;
  to[PM_TO_TOTAL_ENERGY_J] = total; to[PM_TO_ENERGY_SOURCE_TRAPEZOID] = trapezoid ? 1 : 0;
  to[PM_TO_BOARD_POWER_W] = board_power; to[PM_TO_IDLE_ENERGY_J] = idle_energy;
  to[PM_TO_INCREMENTAL_ENERGY_J] = incremental; to[PM_TO_INCREMENTAL_POWER_W] = incremental_power;
  to[PM_TO_OPS_RATE] = ops_rate; to[PM_TO_BYTE_RATE] = byte_rate;
  to[PM_TO_DEVICE_OPS_RATE] = (!none(operations) && truthy(device_duration) && device_duration > 0) ? operations / device_duration : dnan();
  to[PM_TO_DEVICE_BYTE_RATE] = (!none(logical_bytes) && truthy(device_duration) && device_duration > 0) ? logical_bytes / device_duration : dnan();
  to[PM_TO_COUNTED_OPS] = counted_ops; to[PM_TO_COUNTED_BYTES] = counted_bytes;
  to[PM_TO_EPOCHS] = have_epochs ? E.n_inner : 0; to[PM_TO_EXACT] = exact;
  to[PM_TO_RAIL_ENERGY_J] = rail_energy; to[PM_TO_RAIL_INCREMENTAL_J] = rail_incremental;
  to[PM_TO_RAIL_INCREMENTAL_W] = (!none(rail_incremental) && truthy(duration)) ? rail_incremental / duration : dnan();
  to[PM_TO_POWER_LIMIT_W] = power_limit;
  to[PM_TO_TENSOR_PEAK_TFLOPS] = tensor_peak; to[PM_TO_PEAK_CLOCK_IS_SM] = peak_sm;
  to[PM_TO_TENSOR_UTILIZATION] = (!none(ops_rate) && !none(tensor_peak) && tensor_peak > 0) ? ops_rate / 1e12 / tensor_peak : dnan();
  to[PM_TO_IDLE_FRAC_MEASURED] = (!none(idle_power) && truthy(board_power) && board_power > 0) ? idle_power / board_power : dnan();
  to[PM_TO_IDLE_FRAC_LIMIT] = (!none(idle_power) && truthy(power_limit) && power_limit > 0) ? idle_power / power_limit : dnan();
  to[PM_TO_LIMIT_UTILIZATION] = (!none(board_power) && truthy(power_limit) && power_limit > 0) ? board_power / power_limit : dnan();
  const bool ops_ok = truthy(ops_rate) && ops_rate > 0, bytes_ok = truthy(byte_rate) && byte_rate > 0;
  to[PM_TO_PJ_PER_OP] = (!none(incremental_power) && ops_ok && energy_wl) ? incremental_power / ops_rate * 1e12 : dnan();
  to[PM_TO_PJ_PER_LOGICAL_BYTE] = (!none(incremental_power) && bytes_ok) ? incremental_power / byte_rate * 1e12 : dnan();
  to[PM_TO_TOTAL_PJ_PER_OP] = (!none(board_power) && ops_ok && energy_wl) ? board_power / ops_rate * 1e12 : dnan();
  to[PM_TO_TOTAL_PJ_PER_LOGICAL_BYTE] = (!none(board_power) && bytes_ok) ? board_power / byte_rate * 1e12 : dnan();
  to[PM_TO_TOTAL_PJ_PER_FLOP] = (tensor && !none(board_power) && ops_ok) ? board_power / ops_rate * 1e12 : dnan();
  to[PM_TO_TOTAL_PJ_PER_BIT] = (memory && !none(board_power) && bytes_ok) ? board_power / byte_rate / 8 * 1e12 : dnan();
  to[PM_TO_INC_PJ_PER_FLOP] = (tensor && !none(incremental_power) && ops_ok) ? incremental_power / ops_rate * 1e12 : dnan();
  to[PM_TO_INC_PJ_PER_BIT] = (memory && !none(incremental_power) && bytes_ok) ? incremental_power / byte_rate / 8 * 1e12 : dnan();
  to[PM_TO_BASE_CLOCK_MATCHED] = clock_matched; to[PM_TO_BASE_TEMP_MATCHED] = temp_matched;
  to[PM_TO_BASE_CAP_MATCHED] = cap_matched; to[PM_TO_BASE_STATE_MATCHED] = !state_mismatch;
  to[PM_TO_BASE_SM_COMPARED] = base_sm; to[PM_TO_BASE_ENF_COMPARED] = enf_compared; to[PM_TO_BASE_PSTATE_COMPARED] = pst_compared;
  to[PM_TO_THROTTLE_MASK] = thr;
  to[PM_TO_VALID] = valid; to[PM_TO_BASELINE_VALID] = baseline_valid; to[PM_TO_IDLE_INC_ELIGIBLE] = idle_inc_eligible;
  if (has_control) {
    const double* ctl = S.po[PM_CONTROL];
    const double cidle = idle_at(pre, post, ctl, PM_PO_POWER_W), cp = ctl[PM_PO_POWER_W];
    to[PM_TO_CONTROL_INC_POWER_W] = (!none(cp) && !none(cidle)) ? cp - cidle : dnan();
  }

  // ---- paired active reference (analysis.py:292-423) -----------------------
  double contrast = dnan();
  bool paired_eligible = false;
  double ref_slots = dnan();
  if (!has_ref) {
    pair |= 1ull << PM_IP_MISSING_REFERENCE_PHASE;
  } else {
    const uint32_t rf = S.pf[PM_REFERENCE];
    pair |= phase_issue_bits(rf) << PM_IP_R_MISSING_PHASE;
    const EpochResult& RE = S.ep[1];
    if (RE.issue >= 0) pair |= 1ull << (PM_IP_REP_PHASE_WINDOW + RE.issue);
    const bool ref_have = RE.n_inner > 0 && RE.issue < 0;
    if (!ref_have || !RE.exact) pair |= 1ull << PM_IP_REF_WINDOW_UNVERIFIED;
    const int nsel_ref = none(ref[PM_PO_SAMPLES]) ? 0 : (int)ref[PM_PO_SAMPLES];
    for (int k = 0; k < (paired_sm ? 3 : 2); ++k) {
      const double active = mea[med_slot[k]], baseline = ref[med_slot[k]];
      to[PM_TO_PAIRED_D_GFX + k] = (!none(active) && !none(baseline)) ? active - baseline : dnan();
      if (none(active) || none(baseline) || nsel_ref == 0 || scan_ref[k]) pair |= 1ull << (PM_IP_STATE_GFX + k);
    }
    {
      const double active = mea[PM_PO_TEMP_MED], baseline = ref[PM_PO_TEMP_MED];
      to[PM_TO_PAIRED_D_TEMP] = (!none(active) && !none(baseline)) ? active - baseline : dnan();
      if (none(active) || none(baseline) || nsel_ref == 0 || scan_ref[3]) pair |= 1ull << PM_IP_STATE_TEMP;
    }
    to[PM_TO_PAIRED_SM_COMPARED] = paired_sm;
    if (rf & ((1u << PM_PF_THROTTLE_MISSING) | (1u << PM_PF_THROTTLE_ACTIVE))) pair |= 1ull << PM_IP_REF_THROTTLE;
    if (rf & (1u << PM_PF_NO_COMPUTE_INV)) pair |= 1ull << PM_IP_REF_INV_COMPUTE;
    if (rf & (1u << PM_PF_NO_GRAPHICS_INV)) pair |= 1ull << PM_IP_REF_INV_GRAPHICS;
    if (rf & (1u << PM_PF_REF_FOREIGN)) pair |= 1ull << PM_IP_REF_FOREIGN;
    // caps over treatment + reference selected samples
    {
      const double n_none = (none(mea[PM_PO_PLIMIT_NONE]) ? 0 : mea[PM_PO_PLIMIT_NONE]) + (none(ref[PM_PO_PLIMIT_NONE]) ? 0 : ref[PM_PO_PLIMIT_NONE]);
      const double n_fin = (none(mea[PM_PO_PLIMIT_FIN]) ? 0 : mea[PM_PO_PLIMIT_FIN]) + (none(ref[PM_PO_PLIMIT_FIN]) ? 0 : ref[PM_PO_PLIMIT_FIN]);
      const double mn = fmin(none(mea[PM_PO_PLIMIT_MIN]) ? dinf() : mea[PM_PO_PLIMIT_MIN], none(ref[PM_PO_PLIMIT_MIN]) ? dinf() : ref[PM_PO_PLIMIT_MIN]);
      const double mx = fmax(none(mea[PM_PO_PLIMIT_MAX]) ? -dinf() : mea[PM_PO_PLIMIT_MAX], none(ref[PM_PO_PLIMIT_MAX]) ? -dinf() : ref[PM_PO_PLIMIT_MAX]);
      if (n_none + n_fin == 0 || n_none > 0 || mn <= 0) pair |= 1ull << PM_IP_CAP_UNVERIFIED;
      else if (mx - mn > 1e-6) pair |= 1ull << PM_IP_CAP_CHANGED;
    }
    const int fields[2][4] = {{PM_PO_ENF_NONE, PM_PO_ENF_FIN, PM_PO_ENF_MIN, PM_PO_ENF_MAX},
                              {PM_PO_PSTATE_NONE, PM_PO_PSTATE_FIN, PM_PO_PSTATE_MIN, PM_PO_PSTATE_MAX}};
    for (int g = 0; g < 2; ++g) {
      const int* F = fields[g];
      const double an = none(mea[F[0]]) ? 0 : mea[F[0]], af = none(mea[F[1]]) ? 0 : mea[F[1]];
      const double bn = none(ref[F[0]]) ? 0 : ref[F[0]], bf = none(ref[F[1]]) ? 0 : ref[F[1]];
      const bool a_only_none = an > 0 && af == 0, b_only_none = bn > 0 && bf == 0;
      if (!a_only_none || !b_only_none) {
        const bool a_single = an == 0 && af > 0 && mea[F[2]] == mea[F[3]];
        const bool b_single = bn == 0 && bf > 0 && ref[F[2]] == ref[F[3]];
        if (an > 0 || bn > 0 || !a_single || !b_single || mea[F[2]] != ref[F[2]]) pair |= 1ull << (g ? PM_IP_STATE_PSTATE : PM_IP_STATE_ENF);
      }
    }
    const double reference_power = ref[PM_PO_POWER_W];
    contrast = (!none(board_power) && !none(reference_power)) ? board_power - reference_power : dnan();
    if (none(contrast)) pair |= 1ull << PM_IP_POWER_UNAVAILABLE;
    else if (contrast <= 0 && !sfu) pair |= 1ull << PM_IP_NONPOSITIVE_CONTRAST;
    paired_eligible = valid && exact && pair == 0 && !(tflags & PM_T_HOST_PAIRED);
    to[PM_TO_PAIRED_POWER_W] = contrast;
    to[PM_TO_PAIRED_ENERGY_J] = (!none(contrast) && truthy(duration)) ? contrast * duration : dnan();
    to[PM_TO_REF_POWER_W] = reference_power;
    to[PM_TO_REF_DURATION_S] = ref[PM_PO_DURATION_S];
    to[PM_TO_REF_TOTAL_ENERGY_J] = !none(ref[PM_PO_COUNTER_J]) ? ref[PM_PO_COUNTER_J] : ref[PM_PO_ENERGY_J];
    to[PM_TO_REF_EPOCHS] = ref_have ? RE.n_inner : 0; to[PM_TO_REF_EXACT] = ref_have && RE.exact;
    if (sfu) {
      ref_slots = ref_have ? RE.slots : dnan();
      to[PM_TO_REF_SLOTS] = ref_slots;
      to[PM_TO_REF_SLOTS_RATE] = (!none(ref_slots) && truthy(ref[PM_PO_DURATION_S])) ? ref_slots / ref[PM_PO_DURATION_S] : dnan();
    }
    to[PM_TO_PAIRED_PJ_PER_FLOP] = (tensor && !none(contrast) && ops_ok) ? contrast / ops_rate * 1e12 : dnan();
    to[PM_TO_PAIRED_PJ_PER_BIT] = (memory && !none(contrast) && bytes_ok) ? contrast / byte_rate / 8 * 1e12 : dnan();
    const double t_idle = idle_at(pre, post, mea, PM_PO_POWER_W), r_idle = idle_at(pre, post, ref, PM_PO_POWER_W);
    to[PM_TO_PAIRED_DRIFT_ADJUSTED_W] = (idle_inc_eligible && !none(board_power) && !none(t_idle) && !none(reference_power) && !none(r_idle))
        ? (board_power - t_idle) - (reference_power - r_idle) : dnan();
  }
  to[PM_TO_PAIRED_ELIGIBLE] = paired_eligible;

  // ---- SFU and nonlinear normalisation (analysis.py:999-1040) --------------
  double sfu_rate = dnan();
  if (sfu) {
    sfu_rate = ((tflags & PM_T_SFU_CONTRACT_OK) && exact && ops_ok) ? ops_rate : dnan();
    to[PM_TO_SFU_RATE] = sfu_rate;
    to[PM_TO_SFU_COUNTED] = !none(sfu_rate) ? counted_ops : dnan();
    to[PM_TO_SFU_TOTAL_PJ] = (!none(board_power) && truthy(sfu_rate)) ? board_power / sfu_rate * 1e12 : dnan();
    to[PM_TO_SFU_INC_PJ] = (!none(incremental_power) && truthy(sfu_rate)) ? incremental_power / sfu_rate * 1e12 : dnan();
    to[PM_TO_SFU_PAIRED_PJ] = (!none(contrast) && truthy(sfu_rate)) ? contrast / sfu_rate * 1e12 : dnan();
    to[PM_TO_PJ_PER_OP] = dnan(); to[PM_TO_TOTAL_PJ_PER_OP] = dnan();
  }
  const double element_rate = (nonlinear && (tflags & PM_T_NONLINEAR_OK) && exact && ops_ok) ? ops_rate : dnan();
  const double width = (tflags & PM_T_ROWWISE) ? ts[PM_TS_ROW_WIDTH] : dnan();
  const double row_rate = (truthy(element_rate) && truthy(width)) ? element_rate / width : dnan();
  to[PM_TO_ELEMENT_RATE] = element_rate; to[PM_TO_ROW_RATE] = row_rate;
  to[PM_TO_COUNTED_ELEMENTS] = truthy(element_rate) ? counted_ops : dnan();
  if (nonlinear && none(element_rate)) { to[PM_TO_PJ_PER_OP] = dnan(); to[PM_TO_TOTAL_PJ_PER_OP] = dnan(); }
  {
    const double powers[3] = {board_power, incremental_power, contrast};
    for (int k = 0; k < 3; ++k) {
      to[PM_TO_PJ_ELEMENT_TOTAL + k] = (!none(powers[k]) && truthy(element_rate)) ? powers[k] / element_rate * 1e12 : dnan();
      to[PM_TO_PJ_ROW_TOTAL + k] = (!none(powers[k]) && truthy(row_rate)) ? powers[k] / row_rate * 1e12 : dnan();
    }
  }

  // ---- outputs ----------------------------------------------------------------
  uint64_t* ib = R.issue_bits + (size_t)trial * PM_ISSUE_WORDS;
  ib[0] = iss; ib[1] = base; ib[2] = pair; ib[3] = warn;
  R.valid[trial] = valid;
  double* m = R.metrics + (size_t)trial * PM_N_METRICS;   // filled with None above
  m[PM_M_board_power_w] = board_power;
  m[PM_M_idle_power_w] = idle_power;
  m[PM_M_incremental_power_w] = incremental_power;
  m[PM_M_throughput_ops_s] = ops_rate;
  m[PM_M_throughput_bytes_s] = byte_rate;
  m[PM_M_pj_per_op] = to[PM_TO_PJ_PER_OP];
  m[PM_M_pj_per_logical_byte] = to[PM_TO_PJ_PER_LOGICAL_BYTE];
  m[PM_M_total_pj_per_op] = to[PM_TO_TOTAL_PJ_PER_OP];
  m[PM_M_total_pj_per_logical_byte] = to[PM_TO_TOTAL_PJ_PER_LOGICAL_BYTE];
  m[PM_M_memory_rail_power_w] = mea[PM_PO_MEMORY_POWER_W];
  m[PM_M_memory_rail_incremental_power_w] = to[PM_TO_RAIL_INCREMENTAL_W];
  m[PM_M_graphics_clock_mhz] = mea[PM_PO_GFX_MED];
  m[PM_M_sm_clock_mhz] = mea[PM_PO_SM_MED];
  m[PM_M_memory_clock_mhz] = mea[PM_PO_MEM_MED];
  m[PM_M_temperature_c] = mea[PM_PO_TEMP_MED];
  m[PM_M_idle_fraction_of_measured_power] = to[PM_TO_IDLE_FRAC_MEASURED];
  m[PM_M_idle_fraction_of_power_limit] = to[PM_TO_IDLE_FRAC_LIMIT];
  m[PM_M_power_limit_utilization] = to[PM_TO_LIMIT_UTILIZATION];
  m[PM_M_tensor_peak_tflops_at_achieved_clock] = tensor_peak;
  m[PM_M_tensor_utilization_vs_dense_clock_peak] = to[PM_TO_TENSOR_UTILIZATION];
  m[PM_M_total_pj_per_flop] = to[PM_TO_TOTAL_PJ_PER_FLOP];
  m[PM_M_total_pj_per_logical_bit] = to[PM_TO_TOTAL_PJ_PER_BIT];
  m[PM_M_operational_idle_increment_power_w] = incremental_power;
  m[PM_M_operational_idle_increment_energy_j] = incremental;
  m[PM_M_operational_idle_increment_pj_per_flop] = to[PM_TO_INC_PJ_PER_FLOP];
  m[PM_M_operational_idle_increment_pj_per_logical_bit] = to[PM_TO_INC_PJ_PER_BIT];
  m[PM_M_paired_active_reference_power_w] = to[PM_TO_PAIRED_POWER_W];
  m[PM_M_paired_active_reference_energy_j] = to[PM_TO_PAIRED_ENERGY_J];
  m[PM_M_paired_active_reference_pj_per_flop] = to[PM_TO_PAIRED_PJ_PER_FLOP];
  m[PM_M_paired_active_reference_pj_per_logical_bit] = to[PM_TO_PAIRED_PJ_PER_BIT];
  m[PM_M_throughput_elements_s] = element_rate;
  m[PM_M_throughput_rows_s] = row_rate;
  m[PM_M_total_pj_per_element] = to[PM_TO_PJ_ELEMENT_TOTAL];
  m[PM_M_total_pj_per_row] = to[PM_TO_PJ_ROW_TOTAL];
  m[PM_M_operational_idle_increment_pj_per_element] = to[PM_TO_PJ_ELEMENT_INC];
  m[PM_M_operational_idle_increment_pj_per_row] = to[PM_TO_PJ_ROW_INC];
  m[PM_M_paired_active_reference_pj_per_element] = to[PM_TO_PJ_ELEMENT_PAIRED];
  m[PM_M_paired_active_reference_pj_per_row] = to[PM_TO_PJ_ROW_PAIRED];
  if (sfu) {
    m[PM_M_throughput_sfu_instructions_s] = sfu_rate;
    m[PM_M_total_pj_per_instruction] = to[PM_TO_SFU_TOTAL_PJ];
    m[PM_M_operational_idle_increment_pj_per_instruction] = to[PM_TO_SFU_INC_PJ];
    m[PM_M_paired_active_reference_pj_per_instruction] = to[PM_TO_SFU_PAIRED_PJ];
    m[PM_M_sfu_reference_delta_pj_per_instruction] = to[PM_TO_SFU_PAIRED_PJ];
    m[PM_M_sfu_reference_delta_power_w] = has_ref ? contrast : dnan();
    m[PM_M_active_reference_counted_loop_slots] = to[PM_TO_REF_SLOTS];
    m[PM_M_active_reference_loop_slots_s] = to[PM_TO_REF_SLOTS_RATE];
  }
  m[PM_M_active_reference_duration_s] = has_ref ? ref[PM_PO_DURATION_S] : dnan();
  if (X.n_ranks > 0) deliver_rows(X, trial, m, valid, gridDim.x);
}

}  // namespace pm

// ---------------------------------------------------------------------------
// Host launcher (called from capi.cu).
namespace pm {
int launch_analyze(const pm_trials& T, const pm_policy& P, const pm_trial_results& R, int max_covering,
                   double* gscratch, cudaStream_t stream, size_t* scratch_bytes_needed, const pm_peer_rows* rows) {
  int SP = 32;
  while (SP < max_covering + 1) SP <<= 1;
  const size_t smem = (size_t)kTileColumns * SP * sizeof(double);
  const bool use_global = smem > kSmemSortBytes;
  if (scratch_bytes_needed) *scratch_bytes_needed = use_global ? (size_t)T.n_trials * smem : 0;
  if (use_global && !gscratch) return 1;  // caller must supply scratch
  if (T.n_trials == 0) return 0;
  const size_t dyn = use_global ? 0 : smem;
  // The kernel's static shared memory, for the opt-in check.
  static size_t static_bytes = [] {
    cudaFuncAttributes attr{};
    return cudaFuncGetAttributes(&attr, analyze_kernel) == cudaSuccess ? attr.sharedSizeBytes : size_t(48 * 1024);
  }();
  static std::atomic<int> limits[kMaxDevices];
  ensure_dynamic_smem(analyze_kernel, static_bytes, dyn, limits);
  pm_peer_rows X{};
  if (rows) X = *rows;
  analyze_kernel<<<T.n_trials, kThreads, dyn, stream>>>(T, P, R, SP, use_global ? gscratch : nullptr, X);
  return 0;
}
}  // namespace pm
