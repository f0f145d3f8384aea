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

// CPython 3.12's float sum(): the first term is added to int 0, then
// Neumaier's compensated summation (Neumaier 1974) over the rest, with the
// compensation added once at the end when it is nonzero and finite.
struct NeumaierSum {
  double f = 0.0, c = 0.0;
  bool started = false;
  __device__ __forceinline__ void add(double x) {
    if (!started) { f = 0.0 + x; started = true; return; }
    double t = f + x;
    if (fabs(f) >= fabs(x)) c += (f - t) + x;
    else c += (x - t) + f;
    f = t;
  }
  __device__ __forceinline__ double result() const {
    double r = f;
    if (c != 0.0 && isfinite(c)) r += c;
    return r;
  }
};

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

}  // namespace pm
