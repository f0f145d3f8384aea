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
// step is branch-free so a long sum pipelines on its one dependent add.
struct NeumaierSum {
  double f = 0.0, c = 0.0;
  __device__ __forceinline__ void add(double x) {
    const double t = f + x;
    c += fabs(f) >= fabs(x) ? (f - t) + x : (x - t) + f;
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

// CTA-wide ascending bitonic sort of the arrays base + cols[c]*stride
// (c < ncols), each of length P (a power of two, P <= stride).  +inf pads
// and marks excluded values so finite values lead.
__device__ inline void bitonic_sort_columns(double* base, int stride, const int* cols, int ncols, int P) {
  const int half = P >> 1;
  const int lg_half = 31 - __clz(half);
  const int pairs = half * ncols;
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int q = threadIdx.x; q < pairs; q += blockDim.x) {
        const int a = q >> lg_half, p = q & (half - 1);
        const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1));
        double* v = base + (size_t)cols[a] * stride;
        const bool ascending = (i & k) == 0;
        const double x = v[i], y = v[i + j];
        if ((x > y) == ascending) { v[i] = y; v[i + j] = x; }
      }
      __syncthreads();
    }
  }
}

// CTA-wide ascending bitonic sort of v[0, P) (P a power of two, at most
// E * blockDim.x) with the values in registers: thread t holds elements
// [t*E, t*E + E).  Exchanges at distance j < E stay inside a thread, j < 32*E
// are warp shuffles, and only j >= 32*E go through `xchg` (P doubles of
// shared memory) with a CTA barrier, so P = 512 on 256 threads needs 6
// barrier stages instead of 45.  All threads of the CTA call it.
// Up to kSortBatch columns sorted together by cta_register_sort_batch.
constexpr int kSortBatch = 3;

// The compare-exchanges of one bitonic stage between a thread's own
// elements (distance J < E).
template <int E, int J>
__device__ __forceinline__ void register_exchange(double* r, int t, int k) {
  if (J >= E) return;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    if (e & J) continue;
    const bool ascending = ((t * E + e) & k) == 0;
    const double a = r[e], b = r[e | J];
    if ((a > b) == ascending) { r[e] = b; r[e | J] = a; }
  }
}

template <int E>
__device__ void cta_register_sort(double* v, int P, double* xchg) {
  const int t = threadIdx.x;
  double r[E];
#pragma unroll
  for (int e = 0; e < E; ++e) r[e] = t * E + e < P ? v[t * E + e] : dinf();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j < E) {
        // compile-time distances keep r[] in registers
        if (j == 1) register_exchange<E, 1>(r, t, k);
        else if (j == 2) register_exchange<E, 2>(r, t, k);
        else register_exchange<E, 4>(r, t, k);
      } else if (j < 32 * E) {
        const int m = j / E;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const double other = __shfl_xor_sync(0xffffffffu, r[e], m);
          const int i = t * E + e;
          const bool keep_low = ((i & j) == 0) == ((i & k) == 0);
          const double a = r[e];
          const double low = a <= other ? a : other, high = a <= other ? other : a;
          r[e] = keep_low ? low : high;
        }
      } else {
        __syncthreads();
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (t * E + e < P) xchg[t * E + e] = r[e];
        __syncthreads();
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int i = t * E + e;
          if (i >= P) continue;
          const double other = xchg[i ^ j];
          const bool keep_low = ((i & j) == 0) == ((i & k) == 0);
          const double a = r[e];
          const double low = a <= other ? a : other, high = a <= other ? other : a;
          r[e] = keep_low ? low : high;
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < E; ++e)
    if (t * E + e < P) v[t * E + e] = r[e];
  __syncthreads();
}

// cta_register_sort on ncols (<= kSortBatch) columns at once: column c is
// base + cols[c] * stride, its exchange buffer xchg + c * xstride.  The
// columns' stages interleave, so their shuffle latencies overlap and they
// share one set of CTA barriers.  All threads of the CTA call it.
template <int E>
__device__ __forceinline__ void cta_register_sort_batch(double* base, int stride, const int* cols, int ncols, int P, double* xchg,
                                        int xstride) {
  const int t = threadIdx.x;
  double r[kSortBatch][E];
#pragma unroll
  for (int c = 0; c < kSortBatch; ++c)
#pragma unroll
    for (int e = 0; e < E; ++e)
      r[c][e] = (c < ncols && t * E + e < P) ? base[(size_t)cols[c] * stride + t * E + e] : dinf();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j < E) {
#pragma unroll
        for (int c = 0; c < kSortBatch; ++c) {
          if (c >= ncols) continue;
          if (j == 1) register_exchange<E, 1>(r[c], t, k);
          else if (j == 2) register_exchange<E, 2>(r[c], t, k);
          else register_exchange<E, 4>(r[c], t, k);
        }
      } else if (j < 32 * E) {
        const int m = j / E;
#pragma unroll
        for (int c = 0; c < kSortBatch; ++c) {
          if (c >= ncols) continue;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const double other = __shfl_xor_sync(0xffffffffu, r[c][e], m);
            const int i = t * E + e;
            const bool keep_low = ((i & j) == 0) == ((i & k) == 0);
            const double a = r[c][e];
            const double low = a <= other ? a : other, high = a <= other ? other : a;
            r[c][e] = keep_low ? low : high;
          }
        }
      } else {
        __syncthreads();
#pragma unroll
        for (int c = 0; c < kSortBatch; ++c) {
          if (c >= ncols) continue;
#pragma unroll
          for (int e = 0; e < E; ++e)
            if (t * E + e < P) xchg[(size_t)c * xstride + t * E + e] = r[c][e];
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < kSortBatch; ++c) {
          if (c >= ncols) continue;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const int i = t * E + e;
            if (i >= P) continue;
            const double other = xchg[(size_t)c * xstride + (i ^ j)];
            const bool keep_low = ((i & j) == 0) == ((i & k) == 0);
            const double a = r[c][e];
            const double low = a <= other ? a : other, high = a <= other ? other : a;
            r[c][e] = keep_low ? low : high;
          }
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kSortBatch; ++c) {
    if (c >= ncols) continue;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (t * E + e < P) base[(size_t)cols[c] * stride + t * E + e] = r[c][e];
  }
  __syncthreads();
}

// This thread's share of the distinct values in the sorted prefix v[0, n),
// summed over its warp (every lane returns the warp's count).
__device__ inline int warp_share_distinct(const double* v, int n) {
  int d = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) d += (i == 0 || v[i] != v[i - 1]);
  for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  return d;
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

}  // namespace pm
