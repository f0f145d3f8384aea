// Group medians and percentile-bootstrap intervals on sm_100a, one CTA per group.
//
// Restates summarize's group loop (analysis.py:1455-1470) and _median_ci
// (analysis.py:1096-1101):
//   values = finite metric values of the group's valid repeats, in bucket order
//   median = statistics.median(values)
//   ci     = sorted(median(rng.choices(values, k=n)) for _ in range(B))[lo], [hi]
//            with rng = random.Random(seed), lo = 25B/1000-1, hi = 975B/1000-1
// The generator is MT19937 seeded by init_by_array over the 32-bit words of
// the seed (Matsumoto & Nishimura 1998 reference algorithm, as CPython's
// random_seed applies it); choices() draws floor(random()*n) with
// random() = ((w0>>5)*2^26 + (w1>>6)) / 2^53 (CPython Lib/random.py).  Each
// group's stream is produced 624 words per twist by the whole CTA and consumed
// resample by resample in stream order, so every index equals CPython's.
//
// The order statistics are exact without sorting B medians: a resample's
// median depends only on the multiset of drawn indices, so for n <= 7 the
// CTA histograms multisets (C(2n-1, n) <= 1716 bins) and then, per metric,
// folds bins into (rank_a, rank_b) median pairs whose values are sorted once.
// For n >= 8 each draw's median rank pair is binned directly per metric from
// an index stream kept in global scratch.
#include "pmb200.h"
#include "pm_layout.h"
#include "pm_device.cuh"
#include "pm_capi.h"

namespace pm {

constexpr int kBootThreads = 256;
constexpr int kMtN = 624, kMtM = 397;
constexpr int kHistMaxN = 7;            // multiset histogram path
constexpr int kMaxBins = 1716;          // C(13, 7)
constexpr int kDirectMaxN = 128;        // direct path limit
constexpr int kRing = 3 * kMtN;      // block b in slot b % 3: the two newest stay readable

__constant__ uint32_t c_mt_init[kMtN];  // init_genrand(19650218), filled by the host
__constant__ uint32_t c_binom[16][16];  // C(a, b)

__device__ __forceinline__ uint32_t temper(uint32_t y) {
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}
__device__ __forceinline__ uint32_t twist_one(uint32_t cur, uint32_t next, uint32_t far) {
  const uint32_t y = (cur & 0x80000000u) | (next & 0x7fffffffu);
  return far ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
}

// init_by_array(key, key_len) on a 624-word state (single thread).
__device__ void seed_state(uint32_t* mt, uint64_t seed) {
  for (int i = 0; i < kMtN; ++i) mt[i] = c_mt_init[i];
  uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  const int key_len = (seed >> 32) ? 2 : 1;
  int i = 1, j = 0;
  uint32_t prev = mt[0];
  for (int k = kMtN; k; --k) {
    prev = (mt[i] ^ ((prev ^ (prev >> 30)) * 1664525u)) + key[j] + (uint32_t)j;
    mt[i] = prev;
    ++i; ++j;
    if (i >= kMtN) { mt[0] = prev; i = 1; }
    if (j >= key_len) j = 0;
  }
  for (int k = kMtN - 1; k; --k) {
    prev = (mt[i] ^ ((prev ^ (prev >> 30)) * 1566083941u)) - (uint32_t)i;
    mt[i] = prev;
    ++i;
    if (i >= kMtN) { mt[0] = prev; i = 1; }
  }
  mt[0] = 0x80000000u;
}

// One twist of the MT19937 state by the CTA.  `src` holds the current
// state and `dst` receives the next one (ping-pong buffers), so each of the
// three dependency segments needs a single barrier: segment 1 (i < 227)
// reads only old words, segments 2 and 3 read new words of the segment
// before.  Outputs are tempered as they are produced, into ring[base + i].
__device__ __forceinline__ void twist_block(const uint32_t* src, uint32_t* dst, uint32_t* ring, int base) {
  constexpr int A = kMtN - kMtM;          // 227
  for (int i = threadIdx.x; i < A; i += blockDim.x) {
    const uint32_t v = twist_one(src[i], src[i + 1], src[i + kMtM]);
    dst[i] = v; ring[base + i] = temper(v);
  }
  __syncthreads();
  for (int i = A + threadIdx.x; i < 2 * A; i += blockDim.x) {
    const uint32_t v = twist_one(src[i], src[i + 1], dst[i - A]);
    dst[i] = v; ring[base + i] = temper(v);
  }
  __syncthreads();
  for (int i = 2 * A + threadIdx.x; i < kMtN; i += blockDim.x) {
    const uint32_t v = i < kMtN - 1 ? twist_one(src[i], src[i + 1], dst[i - A])
                                    : twist_one(src[kMtN - 1], dst[0], dst[kMtM - 1]);
    dst[i] = v; ring[base + i] = temper(v);
  }
  __syncthreads();
}

__device__ __forceinline__ int draw_index(uint32_t w0, uint32_t w1, double n) {
  const double r = ((double)(w0 >> 5) * 67108864.0 + (double)(w1 >> 6)) * (1.0 / 9007199254740992.0);
  return (int)floor(r * n);
}

// Rank of a non-decreasing n-tuple over [0, n) among multisets (combinatorial
// number system on b_i = a_i + i, strictly increasing in [0, 2n-1)).
// `binom` is a shared-memory copy of c_binom: lookups here are thread-divergent.
__device__ __forceinline__ int multiset_rank(const int* a, int n, const uint32_t (*binom)[16]) {
  int r = 0;
  for (int i = 0; i < n; ++i) r += binom[a[i] + i][i + 1];
  return r;
}
__device__ void multiset_unrank(int r, int n, int* a, const uint32_t (*binom)[16]) {
  // Largest b_{i} with C(b_i, i+1) <= r, from the top index down.
  int top = 2 * n - 2;
  for (int i = n - 1; i >= 0; --i) {
    int b = top;
    while (binom[b][i + 1] > (uint32_t)r) --b;
    r -= (int)binom[b][i + 1];
    a[i] = b - i;
    top = b - 1;
  }
}

// Dynamic shared memory layout (byte offsets) for a launch.
// One resample of a group with exactly N members: draw N indices from the
// ring, sort them (registers only) and count the multiset.  N <= 7.
template <int N>
__device__ __forceinline__ void histogram_resample(const uint32_t* ring, uint32_t pos, uint32_t* hist,
                                                   const uint32_t (*binom)[16]) {
  int t[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t w0 = ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
    const uint32_t w1 = ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
    t[j] = draw_index(w0, w1, double(N));
  }
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int k = 0; k < N - 1 - i; ++k) {
      const int a = t[k], b = t[k + 1];
      t[k] = min(a, b); t[k + 1] = max(a, b);
    }
  int r = 0;
#pragma unroll
  for (int i = 0; i < N; ++i) r += binom[t[i] + i][i + 1];
  atomicAdd(&hist[r], 1u);
}

struct BootSmem {
  size_t vals, cnt, rank_of, sorted_v, ptab, total;
  __host__ __device__ BootSmem(int M, int mm, bool direct) {
    vals = 0;
    cnt = (size_t)M * mm * sizeof(double);
    rank_of = (cnt + (size_t)M * sizeof(int) + 15) & ~(size_t)15;
    sorted_v = rank_of + kDirectMaxN * sizeof(int);
    ptab = sorted_v + kDirectMaxN * sizeof(double);
    total = direct ? ptab + (size_t)kDirectMaxN * kDirectMaxN * sizeof(uint32_t) : rank_of;
  }
};

__global__ void __launch_bounds__(kBootThreads) bootstrap_kernel(BootArgs A) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ uint32_t mt[2][kMtN];
  __shared__ uint32_t ring[kRing];
  __shared__ uint32_t hist[kMaxBins];
  __shared__ uint32_t binom[16][16];
  __shared__ int n_list[kDirectMaxN + 1];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) binom[i >> 4][i & 15] = c_binom[i >> 4][i & 15];
  __shared__ int n_distinct;
  const int g = blockIdx.x;
  const int m0 = A.offsets[g], m1 = A.offsets[g + 1];
  const int members = m1 - m0;
  const int M = A.n_metrics;
  if (members < 0 || members > A.max_members) {            // caller broke the stated bound: no output
    for (int m = threadIdx.x; m < M; m += blockDim.x)
      A.medians[(size_t)g * M + m] = A.lo[(size_t)g * M + m] = A.hi[(size_t)g * M + m] = dnan();
    return;
  }
  const BootSmem L(M, A.max_members, A.max_members > kHistMaxN);
  double* vals = reinterpret_cast<double*>(dsm + L.vals);
  int* cnt = reinterpret_cast<int*>(dsm + L.cnt);
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    int c = 0;
    for (int i = 0; i < members; ++i) {
      const int row = A.member_rows ? A.member_rows[m0 + i] : m0 + i;
      if (A.member_valid && !A.member_valid[row]) continue;
      const double v = A.values[(size_t)row * M + m];
      if (!none(v)) vals[m * A.max_members + c++] = v;
    }
    cnt[m] = c;
    double tmp[64];
    double med = dnan();
    if (c > 0 && c <= 64) {
      for (int i = 0; i < c; ++i) tmp[i] = vals[m * A.max_members + i];
      insertion_sort(tmp, c);
      med = sorted_median(tmp, c);
    } else if (c > 64) {
      // statistics.median of a long row: selection by counting ranks
      double* row = vals + m * A.max_members;
      double a = dnan(), b = dnan();
      const int want_hi = c / 2, want_lo = (c & 1) ? c / 2 : c / 2 - 1;
      for (int i = 0; i < c; ++i) {
        int less = 0, eq = 0;
        for (int k = 0; k < c; ++k) { less += row[k] < row[i]; eq += row[k] == row[i]; }
        if (less <= want_lo && want_lo < less + eq) a = row[i];
        if (less <= want_hi && want_hi < less + eq) b = row[i];
      }
      med = (c & 1) ? b : (a + b) / 2;
    }
    A.medians[(size_t)g * M + m] = med;
    A.lo[(size_t)g * M + m] = dnan();
    A.hi[(size_t)g * M + m] = dnan();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int k = 0;
    for (int m = 0; m < M; ++m) {
      const int c = cnt[m];
      if (c < 3) continue;
      bool seen = false;
      for (int q = 0; q < k; ++q) seen |= n_list[q] == c;
      if (!seen) n_list[k++] = c;
    }
    n_distinct = k;
  }
  __syncthreads();
  const int B = A.resamples;
  const int lo_idx = (int)((25LL * B) / 1000 - 1), hi_idx = (int)((975LL * B) / 1000 - 1);
  for (int d = 0; d < n_distinct; ++d) {
    const int n = n_list[d];
    const bool histogram = n <= kHistMaxN;
    if (!histogram && n > kDirectMaxN) continue;   // host rejects this before launch
    const int nbins = histogram ? (int)binom[2 * n - 1][n] : 0;
    for (int i = threadIdx.x; i < kMaxBins; i += blockDim.x) hist[i] = 0;
    if (threadIdx.x == 0) seed_state(mt[0], A.seeds[g]);
    __syncthreads();
    const double nd = (double)n;
    const uint32_t words_per_draw = 2u * (uint32_t)n;          // 2nB < 2^32 (B <= 2^24, n <= 128)
    const uint32_t blocks = (uint32_t)((2ull * n * B + kMtN - 1) / kMtN);
    uint32_t next_r = 0;
    uint8_t* stream = A.scratch ? A.scratch + (size_t)g * B * kDirectMaxN : nullptr;
    int slot = 0;                                               // ring slot of the current block
    for (uint32_t blk = 0; blk < blocks; ++blk) {
      twist_block(mt[blk & 1], mt[(blk & 1) ^ 1], ring, slot * kMtN);
      // Words [first, avail) are readable: the previous block and this one.
      const uint32_t avail = (blk + 1) * (uint32_t)kMtN;
      const uint32_t first = blk ? avail - 2 * kMtN : 0;
      const int first_slot = blk ? (slot + 2) % 3 : 0;          // slot of word `first`
      uint32_t r_end = avail / words_per_draw;
      if (r_end > (uint32_t)B) r_end = B;
      for (uint32_t r = next_r + threadIdx.x; r < r_end; r += blockDim.x) {
        uint32_t pos = first_slot * kMtN + (r * words_per_draw - first);
        if (pos >= (uint32_t)kRing) pos -= kRing;
        if (histogram) {
          switch (n) {
            case 3: histogram_resample<3>(ring, pos, hist, binom); break;
            case 4: histogram_resample<4>(ring, pos, hist, binom); break;
            case 5: histogram_resample<5>(ring, pos, hist, binom); break;
            case 6: histogram_resample<6>(ring, pos, hist, binom); break;
            default: histogram_resample<7>(ring, pos, hist, binom); break;
          }
        } else {
          for (int j = 0; j < n; ++j) {
            const uint32_t w0 = ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
            const uint32_t w1 = ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
            stream[(size_t)r * n + j] = (uint8_t)draw_index(w0, w1, nd);
          }
        }
      }
      next_r = r_end;
      slot = slot == 2 ? 0 : slot + 1;
    }
    __syncthreads();
    if (histogram) {
      // Per metric: fold multiset bins into median rank pairs, then select.
      for (int m = threadIdx.x; m < M; m += blockDim.x) {
        if (cnt[m] != n) continue;
        const double* v = vals + m * A.max_members;
        // ranks: stable order of the n values
        int rank_of[kHistMaxN]; double sorted_v[kHistMaxN];
        for (int i = 0; i < n; ++i) {
          int r = 0;
          for (int k = 0; k < n; ++k) r += (v[k] < v[i]) || (v[k] == v[i] && k < i);
          rank_of[i] = r; sorted_v[r] = v[i];
        }
        uint32_t pairs[kHistMaxN][kHistMaxN];
        for (int a2 = 0; a2 < n; ++a2) for (int b2 = 0; b2 < n; ++b2) pairs[a2][b2] = 0;
        for (int bin = 0; bin < nbins; ++bin) {
          const uint32_t c = hist[bin];
          if (!c) continue;
          int ms[kHistMaxN], rk[kHistMaxN];
          multiset_unrank(bin, n, ms, binom);
          for (int i = 0; i < n; ++i) rk[i] = rank_of[ms[i]];
          for (int i = 1; i < n; ++i) { int x = rk[i], k = i - 1; while (k >= 0 && rk[k] > x) { rk[k + 1] = rk[k]; --k; } rk[k + 1] = x; }
          const int ra = (n & 1) ? rk[n / 2] : rk[n / 2 - 1];
          const int rb = rk[n / 2];
          pairs[ra][rb] += c;
        }
        double cv[kHistMaxN * kHistMaxN]; uint32_t cc[kHistMaxN * kHistMaxN]; int nc = 0;
        for (int a2 = 0; a2 < n; ++a2)
          for (int b2 = a2; b2 < n; ++b2)
            if (pairs[a2][b2]) {
              cv[nc] = (n & 1) ? sorted_v[a2] : (sorted_v[a2] + sorted_v[b2]) / 2;
              cc[nc++] = pairs[a2][b2];
            }
        for (int i = 1; i < nc; ++i) {
          double x = cv[i]; uint32_t y = cc[i]; int k = i - 1;
          while (k >= 0 && cv[k] > x) { cv[k + 1] = cv[k]; cc[k + 1] = cc[k]; --k; }
          cv[k + 1] = x; cc[k + 1] = y;
        }
        long long cum = 0; double lo = dnan(), hi = dnan();
        for (int i = 0; i < nc; ++i) {
          const long long next = cum + cc[i];
          if (cum <= lo_idx && lo_idx < next) lo = cv[i];
          if (cum <= hi_idx && hi_idx < next) hi = cv[i];
          cum = next;
        }
        A.lo[(size_t)g * M + m] = lo;
        A.hi[(size_t)g * M + m] = hi;
      }
      __syncthreads();
    } else {
      // Direct path: per metric, histogram the median rank pair of every draw.
      int* rank_of = reinterpret_cast<int*>(dsm + L.rank_of);
      double* sorted_v = reinterpret_cast<double*>(dsm + L.sorted_v);
      uint32_t* ptab = reinterpret_cast<uint32_t*>(dsm + L.ptab);   // [n*n] median rank pairs
      for (int m = 0; m < M; ++m) {
        if (cnt[m] != n) continue;
        const double* v = vals + m * A.max_members;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
          int r = 0;
          for (int k = 0; k < n; ++k) r += (v[k] < v[i]) || (v[k] == v[i] && k < i);
          rank_of[i] = r; sorted_v[r] = v[i];
        }
        for (int i = threadIdx.x; i < n * n; i += blockDim.x) ptab[i] = 0;
        __syncthreads();
        for (int r = threadIdx.x; r < B; r += blockDim.x) {
          uint8_t c[kDirectMaxN];
          for (int i = 0; i < n; ++i) c[i] = 0;
          for (int j = 0; j < n; ++j) c[rank_of[stream[(size_t)r * n + j]]]++;
          const int pa = (n & 1) ? n / 2 : n / 2 - 1, pb = n / 2;
          int seen = 0, ra = -1, rb = -1;
          for (int i = 0; i < n && rb < 0; ++i) {
            const int next = seen + c[i];
            if (ra < 0 && pa < next) ra = i;
            if (pb < next) rb = i;
            seen = next;
          }
          atomicAdd(&ptab[ra * n + rb], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
          // Walk candidate values in ascending order by repeated minimum
          // extraction; equal values from different pairs merge their counts.
          long long cum = 0; double lo = dnan(), hi = dnan();
          double last = -dinf(); bool first = true;
          while (true) {
            double best = dinf(); long long count = 0; bool found = false;
            for (int a2 = 0; a2 < n; ++a2) for (int b2 = a2; b2 < n; ++b2) {
              const uint32_t c = ptab[a2 * n + b2];
              if (!c) continue;
              const double val = (n & 1) ? sorted_v[a2] : (sorted_v[a2] + sorted_v[b2]) / 2;
              if ((first || val > last) && (!found || val < best)) { best = val; count = c; found = true; }
              else if (found && val == best && (first || val > last)) count += c;
            }
            if (!found) break;
            const long long next = cum + count;
            if (cum <= lo_idx && lo_idx < next) lo = best;
            if (cum <= hi_idx && hi_idx < next) hi = best;
            cum = next; last = best; first = false;
          }
          A.lo[(size_t)g * M + m] = lo;
          A.hi[(size_t)g * M + m] = hi;
        }
        __syncthreads();
      }
    }
    __syncthreads();
  }
}

// Raw index stream (diagnostic): out[r*n + j] for one seed, by one CTA.
__global__ void resample_indices_kernel(uint64_t seed, int n, int B, int32_t* out) {
  __shared__ uint32_t mt[2][kMtN];
  __shared__ uint32_t ring[kRing];
  if (threadIdx.x == 0) seed_state(mt[0], seed);
  __syncthreads();
  const uint32_t words_per_draw = 2u * (uint32_t)n;
  const uint32_t blocks = (uint32_t)((2ull * n * B + kMtN - 1) / kMtN);
  uint32_t next_r = 0;
  int slot = 0;
  for (uint32_t blk = 0; blk < blocks; ++blk) {
    twist_block(mt[blk & 1], mt[(blk & 1) ^ 1], ring, slot * kMtN);
    const uint32_t avail = (blk + 1) * (uint32_t)kMtN;
    const uint32_t first = blk ? avail - 2 * kMtN : 0;
    const int first_slot = blk ? (slot + 2) % 3 : 0;
    uint32_t r_end = avail / words_per_draw;
    if (r_end > (uint32_t)B) r_end = B;
    for (uint32_t r = next_r + threadIdx.x; r < r_end; r += blockDim.x) {
      uint32_t pos = first_slot * kMtN + (r * words_per_draw - first);
      if (pos >= (uint32_t)kRing) pos -= kRing;
      for (int j = 0; j < n; ++j) {
        const uint32_t w0 = ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
        const uint32_t w1 = ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
        out[(size_t)r * n + j] = draw_index(w0, w1, (double)n);
      }
    }
    next_r = r_end;
    slot = slot == 2 ? 0 : slot + 1;
  }
}

// ---------------------------------------------------------------------------
static bool g_constants_ready[64] = {};

int prepare_bootstrap_constants(int device) {
  if (device < 0 || device >= 64) return 1;
  if (g_constants_ready[device]) return 0;
  uint32_t init[kMtN];
  init[0] = 19650218u;
  for (int i = 1; i < kMtN; ++i) init[i] = 1812433253u * (init[i - 1] ^ (init[i - 1] >> 30)) + (uint32_t)i;
  uint32_t binom[16][16] = {};
  for (int a = 0; a < 16; ++a) {
    binom[a][0] = 1;
    for (int b = 1; b <= a; ++b) binom[a][b] = binom[a - 1][b - 1] + (b <= a - 1 ? binom[a - 1][b] : 0);
  }
  if (cudaMemcpyToSymbol(c_mt_init, init, sizeof(init)) != cudaSuccess) return 2;
  if (cudaMemcpyToSymbol(c_binom, binom, sizeof(binom)) != cudaSuccess) return 2;
  g_constants_ready[device] = true;
  return 0;
}

size_t bootstrap_scratch_bytes(int n_groups, int max_members, int resamples) {
  return max_members > kHistMaxN ? (size_t)n_groups * resamples * kDirectMaxN : 0;
}

int launch_bootstrap(const BootArgs& A, cudaStream_t stream) {
  if (A.n_groups == 0) return 0;
  const size_t smem = BootSmem(A.n_metrics, A.max_members, A.max_members > kHistMaxN).total;
  if (smem > 48 * 1024) cudaFuncSetAttribute(bootstrap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  bootstrap_kernel<<<A.n_groups, kBootThreads, smem, stream>>>(A);
  return 0;
}

int launch_resample_indices(uint64_t seed, int n, int B, int32_t* out, cudaStream_t stream) {
  resample_indices_kernel<<<1, kBootThreads, 0, stream>>>(seed, n, B, out);
  return 0;
}

}  // namespace pm
