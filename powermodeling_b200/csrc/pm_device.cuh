// Device helpers shared by the analysis and bootstrap kernels.
//
// Every floating-point expression here mirrors one in the reference's
// analysis.py in operation order; the files that include this header are
// compiled with --fmad=false so no multiply-add pair is contracted into an FMA
// (CPython rounds every operation separately).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace pm {

__device__ __forceinline__ double dnan() { return __longlong_as_double(0x7ff8000000000000LL); }
__device__ __forceinline__ bool none(double x) { return isnan(x); }
__device__ __forceinline__ double dinf() { return __longlong_as_double(0x7ff0000000000000LL); }

// CPython 3.12's float sum(): Neumaier's compensated summation (Neumaier
// 1974) from 0.0 (the int 0 start, converted) over every term, with the
// compensation added once at the end when it is nonzero and finite.  The
// step is branch-free: the operand of larger magnitude (|f| >= |x| picks f)
// is chosen by an integer compare of the bit patterns without their sign
// bits, which orders magnitudes as the float compare does, so each term
// costs four double adds, (big - t) + small being Neumaier's branch taken.
struct NeumaierSum {
  double f = 0.0, c = 0.0;
  __device__ __forceinline__ void add(double x) {
    const double t = f + x;
    const unsigned long long mf = (unsigned long long)__double_as_longlong(f) & 0x7fffffffffffffffull;
    const unsigned long long mx = (unsigned long long)__double_as_longlong(x) & 0x7fffffffffffffffull;
    const bool f_big = mf >= mx;
    const double big = f_big ? f : x, small = f_big ? x : f;
    c += (big - t) + small;
    f = t;
  }
  __device__ __forceinline__ double result() const {
    double r = f;
    if (c != 0.0 && isfinite(c)) r += c;
    return r;
  }
};

// sum(x[0:n]) in CPython's order, loads hoisted four at a time so only the
// dependent adds remain on the critical path.
__device__ __forceinline__ double neumaier_sum(const double* x, int n) {
  NeumaierSum s;
  int k = 0;
  for (; k + 4 <= n; k += 4) {
    const double a = x[k], b = x[k + 1], c = x[k + 2], d = x[k + 3];
    s.add(a); s.add(b); s.add(c); s.add(d);
  }
  for (; k < n; ++k) s.add(x[k]);
  return s.result();
}

// First index in [lo, hi) with t[i] >= x.
__device__ __forceinline__ int64_t lower_bound(const double* t, int64_t lo, int64_t hi, double x) {
  while (lo < hi) { int64_t mid = lo + ((hi - lo) >> 1); if (t[mid] < x) lo = mid + 1; else hi = mid; }
  return lo;
}
// First index in [lo, hi) with t[i] > x.
__device__ __forceinline__ int64_t upper_bound(const double* t, int64_t lo, int64_t hi, double x) {
  while (lo < hi) { int64_t mid = lo + ((hi - lo) >> 1); if (t[mid] <= x) lo = mid + 1; else hi = mid; }
  return lo;
}

// statistics.median of the first n entries of an ascending array.
__device__ __forceinline__ double sorted_median(const double* a, int n) {
  if (n <= 0) return dnan();
  if (n & 1) return a[n / 2];
  int i = n / 2;
  return (a[i - 1] + a[i]) / 2;
}

// In-register insertion sort for short rows (group medians of repeats).
__device__ __forceinline__ void insertion_sort(double* a, int n) {
  for (int i = 1; i < n; ++i) {
    double v = a[i]; int j = i - 1;
    while (j >= 0 && a[j] > v) { a[j + 1] = a[j]; --j; }
    a[j + 1] = v;
  }
}

// lower_bound (strict = false: first t[i] >= x) or upper_bound (strict =
// true: first t[i] > x) over the sorted t[b, e), by one warp: each round
// probes 32 evenly spaced positions at once, so a segment of n samples takes
// about log32(n) rounds of loads instead of log2(n).  All lanes return it.
__device__ inline int64_t warp_bound(const double* t, int64_t b, int64_t e, double x, bool strict, int lane) {
  int64_t lo = b, hi = e;                       // the answer lies in [lo, hi]
  while (hi - lo > 32) {
    const int64_t step = (hi - lo + 31) / 32;
    const int64_t probe = lo + (int64_t)lane * step;
    const bool past = probe >= hi || (strict ? t[probe] > x : t[probe] >= x);
    const unsigned m = __ballot_sync(0xffffffffu, past);
    if (!m) {
      lo = lo + 31 * step + 1;
    } else {
      const int f = __ffs(m) - 1;
      if (f == 0) return lo;
      const int64_t at = lo + (int64_t)f * step;
      if (at < hi) hi = at;
      lo = lo + (int64_t)(f - 1) * step + 1;
    }
  }
  const int64_t probe = lo + lane;
  const bool past = probe < hi && (strict ? t[probe] > x : t[probe] >= x);
  const unsigned m = __ballot_sync(0xffffffffu, past);
  return m ? lo + (__ffs(m) - 1) : hi;
}

// Key of a non-NaN double whose unsigned order is the values' order (the
// sign bit flipped for positives, every bit for negatives), and back.
__device__ __forceinline__ uint64_t order_key(double v) {
  const uint64_t b = (uint64_t)__double_as_longlong(v);
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}
__device__ __forceinline__ double key_value(uint64_t k) {
  return __longlong_as_double((long long)((k >> 63) ? (k & 0x7fffffffffffffffull) : ~k));
}

// statistics.median of the n finite values of col[0, span) (+inf marks "no
// value"), whose minimum and maximum (cmin < cmax) are known, by one warp.
// Order statistic (n-1)/2 comes from an MSD radix select over the order
// keys, eight bits a pass from the first bit in which cmin and cmax differ
// (every value shares the bits above it), until its bin holds at most 64
// values; those are gathered and ranked by counting, which also gives
// order statistic n/2 unless that one lies past the bin.  Loads are issued
// four at a time ahead of the shared-memory updates they feed.  `hist` is
// 256 words (8-byte aligned) of this warp's shared memory.  All lanes
// return it.
__device__ inline double warp_median(const double* col, int span, int n, double cmin, double cmax, uint32_t* hist) {
  const int lane = threadIdx.x & 31;
  const double inf = dinf();
  const uint64_t kmin = order_key(cmin), kmax = order_key(cmax);
  int shift = ((63 - __clzll((long long)(kmin ^ kmax))) >> 3) << 3;   // digit bits [shift, shift + 8)
  uint64_t prefix = kmin;                                             // bits above the digit are final
  int k = (n - 1) / 2;
  const int rounds = (span + 31) >> 5;
  auto load4 = [&](int r0, double* v) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = ((r0 + u) << 5) + lane;
      v[u] = q < span ? col[q] : inf;
    }
  };
  uint32_t count = 0;
  for (;;) {
    const uint64_t above = shift >= 56 ? 0ull : ~0ull << (shift + 8);
    for (int i = lane; i < 256; i += 32) hist[i] = 0;
    __syncwarp();
    for (int r0 = 0; r0 < rounds; r0 += 4) {
      double v[4];
      load4(r0, v);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint64_t key = order_key(v[u]);
        if (v[u] != inf && ((key ^ prefix) & above) == 0) atomicAdd(&hist[(unsigned)(key >> shift) & 0xffu], 1u);
      }
    }
    __syncwarp();
    // the bin holding rank k: each lane owns eight consecutive bins
    uint32_t c[8], own = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) { c[j] = hist[lane * 8 + j]; own += c[j]; }
    uint32_t incl = own;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    const uint32_t excl = incl - own;
    const unsigned holder = __ballot_sync(0xffffffffu, excl <= (uint32_t)k && (uint32_t)k < incl);
    const int src = __ffs(holder) - 1;
    uint32_t below = excl, bin = 0;
    count = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (count == 0 && (uint32_t)k < below + c[j]) { bin = (uint32_t)(lane * 8 + j); count = c[j]; }
      else if (count == 0) below += c[j];
    }
    bin = __shfl_sync(0xffffffffu, bin, src);
    below = __shfl_sync(0xffffffffu, below, src);
    count = __shfl_sync(0xffffffffu, count, src);
    __syncwarp();                                  // every lane has read hist before it is reused
    prefix = (prefix & above) | ((uint64_t)bin << shift);
    k -= (int)below;
    if (count <= 64 || shift == 0) break;
    shift -= 8;
  }
  double a, b = inf;
  bool have_b = (n & 1) != 0;                      // odd n: order statistic n/2 is a
  if (count <= 64) {
    // gather the bin (every bit >= shift equals the prefix), then rank each
    // gathered value by counting the smaller and equal ones
    double* buf = reinterpret_cast<double*>(hist);
    const uint64_t mask = ~0ull << shift;
    uint32_t base = 0;
    for (int r0 = 0; r0 < rounds; r0 += 4) {
      double v[4];
      load4(r0, v);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool in = v[u] != inf && ((order_key(v[u]) ^ prefix) & mask) == 0;
        const unsigned ballot = __ballot_sync(0xffffffffu, in);
        if (in) buf[base + __popc(ballot & ((1u << lane) - 1u))] = v[u];
        base += __popc(ballot);
      }
    }
    __syncwarp();
    const double x0 = lane < (int)count ? buf[lane] : inf;
    const double x1 = lane + 32 < (int)count ? buf[lane + 32] : inf;
    int less0 = 0, eq0 = 0, less1 = 0, eq1 = 0;
#pragma unroll 4
    for (int i = 0; i < (int)count; ++i) {
      const double y = buf[i];
      less0 += y < x0; eq0 += y == x0;
      less1 += y < x1; eq1 += y == x1;
    }
    __syncwarp();
    auto pick = [&](int r, double* out) -> bool {
      const bool h0 = lane < (int)count && less0 <= r && r < less0 + eq0;
      const bool h1 = lane + 32 < (int)count && less1 <= r && r < less1 + eq1;
      const unsigned m0 = __ballot_sync(0xffffffffu, h0), m1 = __ballot_sync(0xffffffffu, h1);
      if (!(m0 | m1)) return false;
      *out = m0 ? __shfl_sync(0xffffffffu, x0, __ffs(m0) - 1) : __shfl_sync(0xffffffffu, x1, __ffs(m1) - 1);
      return true;
    };
    pick(k, &a);
    if (have_b) b = a;
    else have_b = pick(k + 1, &b);
  } else {
    a = key_value(prefix);                         // all 64 bits fixed: every value in the bin equals it
    if (have_b) b = a;
    else if (k + 1 < (int)count) { b = a; have_b = true; }
  }
  if (!have_b) {
    // order statistic n/2 is the least value above the bin, which ends at a
    for (int r0 = 0; r0 < rounds; r0 += 4) {
      double v[4];
      load4(r0, v);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v[u] > a && v[u] < b) b = v[u];
    }
    for (int o = 16; o; o >>= 1) b = fmin(b, __shfl_xor_sync(0xffffffffu, b, o));
  }
  return (n & 1) ? a : (a + b) / 2;
}

// Insert the bits of finite v (-0.0 as +0.0: equal values share a slot) into
// an open-addressing set of `slots` (a power of two, more than the values
// inserted) 64-bit words cleared to kSetEmpty; true if v was not there yet.
constexpr unsigned long long kSetEmpty = ~0ull;   // a NaN pattern: never a finite value's bits
__device__ __forceinline__ bool set_insert(unsigned long long* set, int slots, double v) {
  const unsigned long long bits = v == 0.0 ? 0ull : (unsigned long long)__double_as_longlong(v);
  unsigned h = (unsigned)((bits * 0x9E3779B97F4A7C15ull) >> 32) & (unsigned)(slots - 1);
  for (int probe = 0; probe < slots; ++probe) {
    const unsigned long long old = atomicCAS(set + h, kSetEmpty, bits);
    if (old == kSetEmpty) return true;
    if (old == bits) return false;
    h = (h + 1) & (unsigned)(slots - 1);
  }
  return false;
}

}  // namespace pm
