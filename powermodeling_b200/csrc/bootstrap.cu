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
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "pmb200.h"
#include "pm_layout.h"
#include "pm_device.cuh"
#include "pm_capi.h"
#include "pmb200_peer.h"

namespace pm {

constexpr int kBootThreads = 256;
constexpr int kPrepThreads = 320;       // the prepare pass: one thread per word pair of a block (312)
constexpr int kMtN = 624, kMtM = 397;
constexpr int kHistMaxN = 7;            // multiset histogram path
constexpr int kMaxBins = 1716;          // C(13, 7)
constexpr int kDirectMaxN = 128;        // direct path limit
constexpr int kRing = 3 * kMtN;      // block b in slot b % 3: the two newest stay readable
constexpr int kFastMaxN = 20;           // direct path in one pass over the draws up to this group size
constexpr int kPtabWords = kDirectMaxN * kDirectMaxN;   // pair-table words (shared by both direct paths)
constexpr int kFastCand = kFastMaxN * (kFastMaxN + 1) / 2;   // distinct median pairs a <= b

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

// init_by_array(key, key_len) on a 624-word state (single thread), with the
// key words of |seed| (one if seed < 2^32, else two).  Both of the reference
// algorithm's loops are unwound into straight index runs (the wrap of i at
// 624 and the alternation of j become explicit), so each step is the
// dependent multiply-xor-add on `prev` and nothing else.
// `init` reads init_genrand(19650218): the constant table (ConstInit) or a
// shared-memory copy of it (the draw pass stages one: the 2.5 KB table does
// not stay in the constant cache across the chain).
struct ConstInit {
  __device__ __forceinline__ uint32_t operator[](int i) const { return c_mt_init[i]; }
};
template <class Init>
__device__ void seed_state(uint32_t* mt, uint64_t seed, Init init) {
  const bool two = (seed >> 32) != 0;
  const uint32_t add0 = (uint32_t)seed;                           // key[0] + 0
  const uint32_t add1 = two ? (uint32_t)(seed >> 32) + 1u : add0;  // key[1] + 1, or key[0] again
  uint32_t prev = init[0];
  // Loop 1 (624 steps): i = 1..623, then i wraps (mt[0] = mt[623]) and i = 1 once more.
#pragma unroll 8
  for (int t = 0; t < kMtN - 1; ++t) {
    prev = (init[1 + t] ^ ((prev ^ (prev >> 30)) * 1664525u)) + ((t & 1) ? add1 : add0);
    mt[1 + t] = prev;
  }
  mt[0] = prev;
  prev = (mt[1] ^ ((prev ^ (prev >> 30)) * 1664525u)) + (((kMtN - 1) & 1) ? add1 : add0);
  mt[1] = prev;
  // Loop 2 (623 steps): i = 2..623, then i wraps (mt[0] = mt[623]) and i = 1.
#pragma unroll 8
  for (int i = 2; i < kMtN; ++i) {
    prev = (mt[i] ^ ((prev ^ (prev >> 30)) * 1566083941u)) - (uint32_t)i;
    mt[i] = prev;
  }
  mt[0] = prev;
  prev = (mt[1] ^ ((prev ^ (prev >> 30)) * 1566083941u)) - 1u;
  mt[1] = prev;
  mt[0] = 0x80000000u;
}

// One twist of the MT19937 state by the CTA.  `src` holds the current
// state and `dst` receives the next one (ping-pong buffers).  Word i < 227
// reads old words only; word i >= 227 reads new word i - 227.  Thread
// t < 227 therefore produces the chain t, t + 227, t + 454 (t < 170) with
// every new operand in its own registers, and the last word (623), which
// also reads new word 0, recomputes that word from the old state: a single
// barrier per twist.  Outputs are tempered as they are produced, into
// ring[base + i].  kBarrier false: the caller places the barrier (after work
// of its own that reads neither `dst` nor ring[base, base + 624)).
template <bool kBarrier = true>
__device__ __forceinline__ void twist_block(const uint32_t* src, uint32_t* dst, uint32_t* ring, int base) {
  constexpr int A = kMtN - kMtM;          // 227
  const int t = threadIdx.x;
  if (t < A) {
    const uint32_t a = twist_one(src[t], src[t + 1], src[t + kMtM]);
    const uint32_t b = twist_one(src[t + A], src[t + A + 1], a);
    dst[t] = a;
    dst[t + A] = b;
    ring[base + t] = temper(a);
    ring[base + t + A] = temper(b);
    if (t < kMtN - 2 * A) {
      const int i = t + 2 * A;
      const uint32_t next = i < kMtN - 1 ? src[i + 1] : twist_one(src[0], src[1], src[kMtM]);
      const uint32_t c = twist_one(src[i], next, b);
      dst[i] = c;
      ring[base + i] = temper(c);
    }
  }
  if (kBarrier) __syncthreads();
}

__device__ __forceinline__ int draw_index(uint32_t w0, uint32_t w1, double n) {
  const double r = ((double)(w0 >> 5) * 67108864.0 + (double)(w1 >> 6)) * (1.0 / 9007199254740992.0);
  return (int)floor(r * n);
}
// For n = 2^p (1 <= p <= 26) random() * n only rescales the 53-bit fraction, so
// it is exact and floor(random() * n) is the top p bits of the first word:
// w0 >> (32 - p).  pow2_shift(n) is that shift, or 0 when n is not such a power.
__device__ __forceinline__ int pow2_shift(int n) { return n >= 2 && (n & (n - 1)) == 0 ? 33 - __ffs(n) : 0; }

// twist_block for n = 2^p: a draw reads the first (even) word of its pair
// alone, so each even word's index goes straight from the twist into the
// stream (draw d0 + i / 2 for word i, kept while below `draws`); odd words are
// neither tempered nor kept, and no ring or conversion pass is needed.  The
// chain t, t + 227, t + 454 alternates parity (227 is odd), so threads 0-127
// take the even t and threads 128-255 the odd t: every warp tempers the same
// words of its chains.  The state sits even words first (word i at
// emit_slot(i)), so a warp's loads and stores of one parity are consecutive.
__device__ __forceinline__ int emit_slot(int i) { return (i & 1) * (kMtN / 2) + (i >> 1); }

template <int kParity>
__device__ __forceinline__ void twist_chain_emit(const uint32_t* src, uint32_t* dst, uint8_t* stream, uint32_t d0,
                                                 uint32_t draws, int shift, int k) {
  constexpr int A = kMtN - kMtM;          // 227
  const int t = 2 * k + kParity;
  auto emit = [&](int i, uint32_t w) {    // i even
    const uint32_t d = d0 + (uint32_t)(i >> 1);
    if (d < draws) stream[d] = (uint8_t)(temper(w) >> shift);
  };
  const uint32_t a = twist_one(src[emit_slot(t)], src[emit_slot(t + 1)], src[emit_slot(t + kMtM)]);
  const uint32_t b = twist_one(src[emit_slot(t + A)], src[emit_slot(t + A + 1)], a);
  dst[emit_slot(t)] = a;
  dst[emit_slot(t + A)] = b;
  if (kParity == 0) emit(t, a); else emit(t + A, b);
  if (t < kMtN - 2 * A) {
    const int i = t + 2 * A;
    const uint32_t next = i < kMtN - 1 ? src[emit_slot(i + 1)]
                                       : twist_one(src[emit_slot(0)], src[emit_slot(1)], src[emit_slot(kMtM)]);
    const uint32_t c = twist_one(src[emit_slot(i)], next, b);
    dst[emit_slot(i)] = c;
    if (kParity == 0) emit(i, c);
  }
}

// Needs blockDim.x >= 256; src and dst in the emit_slot layout.
__device__ __forceinline__ void twist_block_emit(const uint32_t* src, uint32_t* dst, uint8_t* stream, uint32_t d0,
                                                 uint32_t draws, int shift) {
  constexpr int A = kMtN - kMtM;
  const int r = threadIdx.x;
  if (r < 128) {
    if (2 * r < A) twist_chain_emit<0>(src, dst, stream, d0, draws, shift, r);
  } else if (r < 256) {
    if (2 * (r - 128) + 1 < A) twist_chain_emit<1>(src, dst, stream, d0, draws, shift, r - 128);
  }
  __syncthreads();
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

// Dynamic shared memory layout (byte offsets) for a launch.  The histogram
// path (every group has at most kHistMaxN members) folds in shared tables:
// per metric the values in rank order and the member index of each rank, a
// median-pair table per metric, and the index counts of every multiset bin.
struct BootSmem {
  size_t vals, cnt, rank_of, sorted_v, ptab, fold_sorted, fold_index, fold_pairs, bin_counts;
  size_t fast_list, fast_index, fast_sorted, fast_counts, cand_vals, cand_counts, total;
  __host__ __device__ BootSmem(int M, int mm, bool direct) {
    auto up = [](size_t x) { return (x + 15) & ~(size_t)15; };
    vals = 0;
    cnt = (size_t)M * mm * sizeof(double);
    rank_of = up(cnt + (size_t)M * sizeof(int));
    sorted_v = rank_of + kDirectMaxN * sizeof(int);
    ptab = sorted_v + kDirectMaxN * sizeof(double);
    fold_sorted = rank_of;
    fold_index = up(fold_sorted + (size_t)M * kHistMaxN * sizeof(double));
    fold_pairs = up(fold_index + (size_t)M * kHistMaxN);
    bin_counts = up(fold_pairs + (size_t)M * kHistMaxN * kHistMaxN * sizeof(uint32_t));
    // direct path, one pass: active metric list, per-metric rank order and
    // sorted values, per-thread index counts, per-warp candidate lists (twice:
    // as collected and in value order)
    fast_list = up(ptab + (size_t)kPtabWords * sizeof(uint32_t));
    fast_index = up(fast_list + (size_t)M * sizeof(int));
    fast_sorted = up(fast_index + (size_t)M * kFastMaxN);
    fast_counts = up(fast_sorted + (size_t)M * kFastMaxN * sizeof(double));
    cand_vals = up(fast_counts + (size_t)kBootThreads * kFastMaxN);
    cand_counts = up(cand_vals + (size_t)(kBootThreads / 32) * 2 * kFastCand * sizeof(double));
    total = direct ? up(cand_counts + (size_t)(kBootThreads / 32) * 2 * kFastCand * sizeof(uint32_t))
                   : up(bin_counts + (size_t)kMaxBins * kHistMaxN);
  }
};

// Scratch layout: one prepared multiset histogram per group (kMaxBins words),
// then, when the prepare pass streams every group (A.streamed) or a group may
// have more than kHistMaxN members, one index stream per group: B resamples
// of up to max_members one-byte indices, resample r of a count-n draw at
// [r n, r n + n).
__host__ __device__ inline size_t hist_area_bytes(int n_groups) {
  return ((size_t)n_groups * kMaxBins * sizeof(uint32_t) + 255) & ~(size_t)255;
}
__device__ inline uint32_t* prepared_hist(const BootArgs& A, int g) {
  return reinterpret_cast<uint32_t*>(A.scratch) + (size_t)g * kMaxBins;
}
__device__ inline uint8_t* index_stream(const BootArgs& A, int g) {
  return A.streamed || A.max_members > kHistMaxN
             ? A.scratch + hist_area_bytes(A.n_groups) + (size_t)g * A.resamples * A.max_members
             : nullptr;
}

// Shared state of one group's stream.
struct GenShared {
  uint32_t mt[2][kMtN];
  uint32_t mt_seed[kMtN];
  uint32_t ring[kRing];
  uint32_t hist[kMaxBins];
  uint32_t binom[16][16];
};

__device__ __forceinline__ void load_binom(GenShared& sh) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) sh.binom[i >> 4][i & 15] = c_binom[i >> 4][i & 15];
}

// B resamples of n draws from the seeded state in sh.mt_seed, generated and
// consumed block by block in one CTA: multiset counts into sh.hist
// (n <= kHistMaxN, hist cleared here) or raw indices into `stream`
// (n > kHistMaxN).  The finish uses it for a count that was not prepared, and
// the prepare pass when the scratch holds no streams.  All threads call it.
__device__ __forceinline__ void generate_resamples(GenShared& sh, int n, int B, uint8_t* stream) {
  const bool histogram = n <= kHistMaxN;
  if (histogram)
    for (int i = threadIdx.x; i < kMaxBins; i += blockDim.x) sh.hist[i] = 0;
  for (int i = threadIdx.x; i < kMtN; i += blockDim.x) sh.mt[0][i] = sh.mt_seed[i];
  __syncthreads();
  const double nd = (double)n;
  const uint32_t words_per_draw = 2u * (uint32_t)n;          // 2nB < 2^32 (B <= 2^24, n <= 128)
  const uint32_t blocks = (uint32_t)(((uint64_t)B * words_per_draw + kMtN - 1) / kMtN);
  uint32_t next_r = 0;
  int slot = 0;                                               // ring slot of the current block
  for (uint32_t blk = 0; blk < blocks; ++blk) {
    twist_block(sh.mt[blk & 1], sh.mt[(blk & 1) ^ 1], sh.ring, slot * kMtN);
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
          case 3: histogram_resample<3>(sh.ring, pos, sh.hist, sh.binom); break;
          case 4: histogram_resample<4>(sh.ring, pos, sh.hist, sh.binom); break;
          case 5: histogram_resample<5>(sh.ring, pos, sh.hist, sh.binom); break;
          case 6: histogram_resample<6>(sh.ring, pos, sh.hist, sh.binom); break;
          default: histogram_resample<7>(sh.ring, pos, sh.hist, sh.binom); break;
        }
      } else {
        for (int j = 0; j < n; ++j) {
          const uint32_t w0 = sh.ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
          const uint32_t w1 = sh.ring[pos]; if (++pos == (uint32_t)kRing) pos = 0;
          stream[(size_t)r * n + j] = (uint8_t)draw_index(w0, w1, nd);
        }
      }
    }
    next_r = r_end;
    slot = slot == 2 ? 0 : slot + 1;
  }
  __syncthreads();
}

// The group's whole index stream (B n draws, one byte each) from the seeded
// state in sh.mt_seed, with nothing else in the generator's serial chain: each
// pass twists block k into one half of the ring while the threads turn the
// 312 word pairs of block k - 1 (the other half) into draw indices and store
// them, then one barrier.  A draw never straddles two blocks (624 is even),
// so draw d of the stream is pair d mod 312 of block d / 312.  For n = 2^p
// the twist stores the indices itself (twist_block_emit, state in the
// emit_slot layout): one barrier per block and nothing else in the loop.
// Needs blockDim.x >= 312.  All threads call it.
__device__ __forceinline__ void stream_draws(GenShared& sh, int n, int B, uint8_t* stream) {
  constexpr int kPairs = kMtN / 2;
  const int shift = pow2_shift(n);
  for (int i = threadIdx.x; i < kMtN; i += blockDim.x) sh.mt[0][shift ? emit_slot(i) : i] = sh.mt_seed[i];
  __syncthreads();
  const double nd = (double)n;
  const uint32_t draws = (uint32_t)B * (uint32_t)n;
  const uint32_t blocks = (draws + kPairs - 1) / kPairs;
  if (shift) {
    for (uint32_t blk = 0; blk < blocks; ++blk)
      twist_block_emit(sh.mt[blk & 1], sh.mt[(blk & 1) ^ 1], stream, blk * kPairs, draws, shift);
    return;
  }
  const int j = threadIdx.x;
  for (uint32_t blk = 0; blk <= blocks; ++blk) {
    if (blk < blocks) twist_block<false>(sh.mt[blk & 1], sh.mt[(blk & 1) ^ 1], sh.ring, (int)(blk & 1) * kMtN);
    if (blk > 0 && j < kPairs) {
      const uint32_t d = (blk - 1) * kPairs + j;
      const uint32_t* words = sh.ring + ((blk - 1) & 1) * kMtN;
      if (d < draws)
        stream[d] = (uint8_t)(shift ? (int)(words[2 * j] >> shift) : draw_index(words[2 * j], words[2 * j + 1], nd));
    }
    __syncthreads();
  }
}

// Multiset counts of the B resamples of a count-N stream (N <= kHistMaxN)
// into sh.hist: each thread sorts its resamples' indices in registers and
// ranks the multiset; lanes of a warp holding the same rank add once together.
// The stream was written by this CTA and sits in L2: each thread reads the
// indices of kBatch resamples before ranking any of them.
template <int N>
__device__ __forceinline__ void histogram_stream(GenShared& sh, int B, const uint8_t* stream) {
  constexpr int kBatch = 4;
  for (int r0 = 0; r0 < B; r0 += blockDim.x * kBatch) {
    int t[kBatch][N];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int r = r0 + u * blockDim.x + threadIdx.x;
#pragma unroll
      for (int i = 0; i < N; ++i) t[u][i] = r < B ? stream[(size_t)r * N + i] : 0;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int r = r0 + u * blockDim.x + threadIdx.x;
      int rank = -1;
      if (r < B) {
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int k = 0; k < N - 1 - i; ++k) {
            const int a = t[u][k], b = t[u][k + 1];
            t[u][k] = min(a, b); t[u][k + 1] = max(a, b);
          }
        rank = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) rank += (int)sh.binom[t[u][i] + i][i + 1];
      }
      const unsigned live = __ballot_sync(0xffffffffu, rank >= 0);
      if (rank >= 0) {
        const unsigned same = __match_any_sync(live, rank);
        if ((int)(threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&sh.hist[rank], (uint32_t)__popc(same));
      }
    }
  }
}

// Stream generation ahead of the fold: for each group's member count n (the
// count every metric has when all listed members are valid and finite), the
// multiset histogram (n <= kHistMaxN) and, where the scratch holds streams,
// the index stream.  It needs only seeds and group sizes, so it runs while
// the trials are still analysed.  A.streamed: the index stream first (the
// generator's chain alone), then the histogram from it; otherwise the
// resamples are consumed as the blocks are produced.
__global__ void __launch_bounds__(kPrepThreads) bootstrap_prepare_kernel(BootArgs A) {
  __shared__ GenShared sh;
  const int g = blockIdx.x;
  const int n = A.offsets[g + 1] - A.offsets[g];
  if (n < 3 || n > A.max_members || n > kDirectMaxN) return;   // no interval for n < 3 (uniform exit)
  load_binom(sh);
  // The seeding table in shared memory (sh.mt[1] is free until the first twist).
  for (int i = threadIdx.x; i < kMtN; i += blockDim.x) sh.mt[1][i] = c_mt_init[i];
  __syncthreads();
  if (threadIdx.x == 0) seed_state(sh.mt_seed, A.seeds[g], static_cast<const uint32_t*>(sh.mt[1]));
  for (int i = threadIdx.x; i < kMaxBins; i += blockDim.x) sh.hist[i] = 0;
  __syncthreads();
  uint8_t* stream = index_stream(A, g);
  if (A.streamed) {
    stream_draws(sh, n, A.resamples, stream);
    switch (n) {
      case 3: histogram_stream<3>(sh, A.resamples, stream); break;
      case 4: histogram_stream<4>(sh, A.resamples, stream); break;
      case 5: histogram_stream<5>(sh, A.resamples, stream); break;
      case 6: histogram_stream<6>(sh, A.resamples, stream); break;
      case 7: histogram_stream<7>(sh, A.resamples, stream); break;
      default: break;                                          // direct path: the stream is the product
    }
    __syncthreads();
  } else {
    generate_resamples(sh, n, A.resamples, stream);
  }
  if (n <= kHistMaxN) {
    uint32_t* out = prepared_hist(A, g);
    const int nbins = (int)sh.binom[2 * n - 1][n];
    for (int i = threadIdx.x; i < nbins; i += blockDim.x) out[i] = sh.hist[i];
  }
}

__device__ __noinline__ void deliver_groups(const pm_peer_groups& X, const BootArgs& A, int g);

// The finish of one group (the CTA's): medians, fold and intervals.
// kDeliver: the sharded form, which also delivers the group to every rank.
template <bool kDeliver>
__global__ void __launch_bounds__(kBootThreads) bootstrap_kernel(BootArgs A, pm_peer_groups X) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ GenShared sh;
  __shared__ uint32_t n_mask[(kDirectMaxN + 1 + 31) / 32];
  __shared__ int s_active, s_cand[kBootThreads / 32];
  load_binom(sh);
  for (int i = threadIdx.x; i < (kDirectMaxN + 1 + 31) / 32; i += blockDim.x) n_mask[i] = 0;
  __syncthreads();
  const int g = blockIdx.x;
  const int m0 = A.offsets[g], m1 = A.offsets[g + 1];
  const int members = m1 - m0;
  const int M = A.n_metrics;
  if (members < 0 || members > A.max_members) {            // caller broke the stated bound: no output
    for (int m = threadIdx.x; m < M; m += blockDim.x)
      A.medians[(size_t)g * M + m] = A.lo[(size_t)g * M + m] = A.hi[(size_t)g * M + m] = dnan();
    if constexpr (kDeliver) {
      __syncthreads();
      deliver_groups(X, A, g);
    }
    return;
  }
  // Without a prepare pass, one thread of the last warp seeds the generator
  // while the others gather the metric values (every metric's _median_ci
  // starts random.Random(seed) afresh, so one seeded state serves them all).
  if (!A.prepared && threadIdx.x == blockDim.x - 32) seed_state(sh.mt_seed, A.seeds[g], ConstInit{});
  const BootSmem L(M, A.max_members, A.max_members > kHistMaxN);
  double* vals = reinterpret_cast<double*>(dsm + L.vals);
  int* cnt = reinterpret_cast<int*>(dsm + L.cnt);
  // The group's rows (-1: not valid) first, so each metric's value loads are
  // independent of one another.
  __shared__ int s_rows[kDirectMaxN];
  for (int i = threadIdx.x; i < members; i += blockDim.x) {
    const int row = A.member_rows ? A.member_rows[m0 + i] : m0 + i;
    s_rows[i] = (A.member_valid && !A.member_valid[row]) ? -1 : row;
  }
  __syncthreads();
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    int c = 0;
    for (int i0 = 0; i0 < members; i0 += 4) {
      double v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int row = i0 + u < members ? s_rows[i0 + u] : -1;
        v[u] = row >= 0 ? A.values[(size_t)row * M + m] : dnan();
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (!none(v[u])) vals[m * A.max_members + c++] = v[u];
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
    if (c >= 3) atomicOr(&n_mask[c >> 5], 1u << (c & 31));   // intervals need n >= 3
  }
  __syncthreads();
  const int B = A.resamples;
  const int lo_idx = (int)((25LL * B) / 1000 - 1), hi_idx = (int)((975LL * B) / 1000 - 1);
  // The member count first (its stream may be prepared, and a direct-path
  // stream must be consumed before another count reuses the group's area),
  // then every other count in ascending order.
  bool seeded = !A.prepared;
  // The counts present come from the shared mask (read after a barrier, so
  // every thread walks the same list): the member count, then its set bits
  // in ascending order.
  constexpr int kMaskWords = (kDirectMaxN + 1 + 31) / 32;
  uint32_t rest[kMaskWords];
#pragma unroll
  for (int w = 0; w < kMaskWords; ++w) rest[w] = n_mask[w];
  bool member_count_first = members >= 3 && members <= kDirectMaxN && ((rest[members >> 5] >> (members & 31)) & 1u);
  if (member_count_first) rest[members >> 5] &= ~(1u << (members & 31));
  for (;;) {
    int n = -1;
    if (member_count_first) {
      n = members;
      member_count_first = false;
    } else {
#pragma unroll
      for (int w = 0; w < kMaskWords; ++w)
        if (n < 0 && rest[w]) { n = w * 32 + __ffs(rest[w]) - 1; rest[w] &= rest[w] - 1; }
      if (n < 0) break;
    }
    if (n < 3) continue;                                   // counts below 3 carry no interval
    const bool histogram = n <= kHistMaxN;
    const int nbins = histogram ? (int)sh.binom[2 * n - 1][n] : 0;
    uint8_t* stream = index_stream(A, g);
    if (A.prepared && n == members) {
      if (histogram) {
        const uint32_t* prepared = prepared_hist(A, g);
        for (int i = threadIdx.x; i < nbins; i += blockDim.x) sh.hist[i] = prepared[i];
      }
      __syncthreads();
    } else {
      if (!seeded) {
        if (threadIdx.x == 0) seed_state(sh.mt_seed, A.seeds[g], ConstInit{});
        seeded = true;
      }
      __syncthreads();
      generate_resamples(sh, n, B, stream);
    }
    uint32_t* hist = sh.hist;
    const uint32_t (*binom)[16] = sh.binom;
    if (histogram) {
      // Fold the multiset histogram into each metric's median rank pairs, over
      // (metric, bin) items on every thread: a bin's median ranks under a
      // metric follow from the bin's index counts walked in that metric's
      // rank order.
      double* fsorted = reinterpret_cast<double*>(dsm + L.fold_sorted);       // [M][kHistMaxN]
      uint8_t* findex = dsm + L.fold_index;                                   // [M][kHistMaxN]
      uint32_t* fpairs = reinterpret_cast<uint32_t*>(dsm + L.fold_pairs);     // [M][kHistMaxN^2]
      uint8_t* bcounts = dsm + L.bin_counts;                                  // [kMaxBins][kHistMaxN]
      for (int bin = threadIdx.x; bin < nbins; bin += blockDim.x) {
        int ms[kHistMaxN];
        multiset_unrank(bin, n, ms, binom);
        uint8_t* c = bcounts + bin * kHistMaxN;
        for (int i = 0; i < n; ++i) c[i] = 0;
        for (int i = 0; i < n; ++i) c[ms[i]]++;
      }
      for (int m = threadIdx.x; m < M; m += blockDim.x) {
        if (cnt[m] != n) continue;
        const double* v = vals + m * A.max_members;
        for (int i = 0; i < n; ++i) {                  // stable ranks: ties keep member order
          int r = 0;
          for (int k = 0; k < n; ++k) r += (v[k] < v[i]) || (v[k] == v[i] && k < i);
          fsorted[m * kHistMaxN + r] = v[i];
          findex[m * kHistMaxN + r] = (uint8_t)i;
        }
      }
      for (int i = threadIdx.x; i < M * n * n; i += blockDim.x) fpairs[(i / (n * n)) * kHistMaxN * kHistMaxN + i % (n * n)] = 0;
      __syncthreads();
      const int pa = (n & 1) ? n / 2 : n / 2 - 1, pb = n / 2;
      // Each thread takes a run of consecutive (metric, bin) items, metric
      // major: mostly the bins of one metric, whose rank-to-member map it
      // holds in registers; a metric's items fall to a few threads only.
      {
        const int items = M * nbins;
        const int per = (items + (int)blockDim.x - 1) / (int)blockDim.x;
        const int i0 = (int)threadIdx.x * per, i1 = min(items, i0 + per);
        int m = i0 / nbins, bin = i0 - m * nbins, cur = -1;
        bool live = false;
        int id[kHistMaxN];
        uint32_t* pt = fpairs;
        for (int it = i0; it < i1; ++it) {
          if (m != cur) {
            cur = m;
            live = cnt[m] == n;
#pragma unroll
            for (int r = 0; r < kHistMaxN; ++r) id[r] = r < n ? findex[m * kHistMaxN + r] : 0;
            pt = fpairs + m * kHistMaxN * kHistMaxN;
          }
          const uint32_t h = live ? hist[bin] : 0u;
          if (h) {
            const uint8_t* c = bcounts + bin * kHistMaxN;
            int seen = 0, ra = -1, rb = -1;
#pragma unroll
            for (int r = 0; r < kHistMaxN; ++r) {
              if (r < n && rb < 0) {
                seen += c[id[r]];
                if (ra < 0 && pa < seen) ra = r;
                if (pb < seen) rb = r;
              }
            }
            atomicAdd(&pt[ra * n + rb], h);
          }
          if (++bin == nbins) { bin = 0; ++m; }
        }
      }
      __syncthreads();
      // Per metric: the pair values in ascending order with their counts, then
      // the two order statistics of the B resampled medians.
      for (int m = threadIdx.x; m < M; m += blockDim.x) {
        if (cnt[m] != n) continue;
        const double* sv = fsorted + m * kHistMaxN;
        const uint32_t* pt = fpairs + m * kHistMaxN * kHistMaxN;
        double cv[kHistMaxN * (kHistMaxN + 1) / 2]; uint32_t cc[kHistMaxN * (kHistMaxN + 1) / 2]; int nc = 0;
        for (int a2 = 0; a2 < n; ++a2)
          for (int b2 = a2; b2 < n; ++b2)
            if (pt[a2 * n + b2]) {
              const double x = (n & 1) ? sv[a2] : (sv[a2] + sv[b2]) / 2;
              const uint32_t y = pt[a2 * n + b2];
              int k = nc - 1;
              while (k >= 0 && cv[k] > x) { cv[k + 1] = cv[k]; cc[k + 1] = cc[k]; --k; }
              cv[k + 1] = x; cc[k + 1] = y; ++nc;
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
      // Direct path.  The metrics with this count, in order:
      int* flist = reinterpret_cast<int*>(dsm + L.fast_list);
      if (threadIdx.x == 0) {
        int k = 0;
        for (int m = 0; m < M; ++m) if (cnt[m] == n) flist[k++] = m;
        s_active = k;
      }
      __syncthreads();
      const int K = s_active;
      const int pa = (n & 1) ? n / 2 : n / 2 - 1, pb = n / 2;
      if (n <= kFastMaxN && K * n * n <= kPtabWords) {
        // One pass over the draws for every metric: each draw's index counts in
        // the thread's shared row, then each metric's median rank pair by a
        // walk in that metric's rank order.
        uint8_t* fidx = dsm + L.fast_index;                                    // [K][kFastMaxN]
        double* fsv = reinterpret_cast<double*>(dsm + L.fast_sorted);          // [K][kFastMaxN]
        uint32_t* pairs = reinterpret_cast<uint32_t*>(dsm + L.ptab);           // [K][n*n]
        uint8_t* counts = dsm + L.fast_counts + threadIdx.x * kFastMaxN;
        for (int a = threadIdx.x; a < K; a += blockDim.x) {
          const double* v = vals + flist[a] * A.max_members;
          for (int i = 0; i < n; ++i) {                  // stable ranks: ties keep member order
            int r = 0;
            for (int k = 0; k < n; ++k) r += (v[k] < v[i]) || (v[k] == v[i] && k < i);
            fidx[a * kFastMaxN + r] = (uint8_t)i;
            fsv[a * kFastMaxN + r] = v[i];
          }
        }
        for (int i = threadIdx.x; i < K * n * n; i += blockDim.x) pairs[i] = 0;
        __syncthreads();
        for (int r = threadIdx.x; r < B; r += blockDim.x) {
          for (int i = 0; i < n; ++i) counts[i] = 0;
          const uint8_t* draw = stream + (size_t)r * n;
          for (int j = 0; j < n; ++j) counts[draw[j]]++;
          for (int a = 0; a < K; ++a) {
            const uint8_t* idx = fidx + a * kFastMaxN;
            int seen = 0, ra = -1, rb = -1;
            for (int q = 0; q < n && rb < 0; ++q) {
              seen += counts[idx[q]];
              if (ra < 0 && pa < seen) ra = q;
              if (pb < seen) rb = q;
            }
            atomicAdd(&pairs[a * n * n + ra * n + rb], 1u);
          }
        }
        __syncthreads();
        // Per metric, one warp: the distinct pair values in ascending order
        // with their counts (rank by counting), then the two order statistics.
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
        double* cv = reinterpret_cast<double*>(dsm + L.cand_vals) + (size_t)warp * 2 * kFastCand;
        uint32_t* cc = reinterpret_cast<uint32_t*>(dsm + L.cand_counts) + (size_t)warp * 2 * kFastCand;
        for (int a = warp; a < K; a += warps) {
          const double* sv = fsv + a * kFastMaxN;
          const uint32_t* pt = pairs + a * n * n;
          if (lane == 0) s_cand[warp] = 0;
          __syncwarp();
          for (int p2 = lane; p2 < n * n; p2 += 32) {
            const int a2 = p2 / n, b2 = p2 - a2 * n;
            if (a2 <= b2 && pt[p2]) {
              const int k = atomicAdd(&s_cand[warp], 1);
              cv[k] = (n & 1) ? sv[a2] : (sv[a2] + sv[b2]) / 2;
              cc[k] = pt[p2];
            }
          }
          __syncwarp();
          const int kc = s_cand[warp];
          for (int i = lane; i < kc; i += 32) {
            const double x = cv[i];
            int rank = 0;
            for (int j = 0; j < kc; ++j) rank += (cv[j] < x) || (cv[j] == x && j < i);
            cv[kFastCand + rank] = x;
            cc[kFastCand + rank] = cc[i];
          }
          __syncwarp();
          if (lane == 0) {
            long long cum = 0; double lo = dnan(), hi = dnan();
            for (int i = 0; i < kc; ++i) {
              const long long next = cum + cc[kFastCand + i];
              if (cum <= lo_idx && lo_idx < next) lo = cv[kFastCand + i];
              if (cum <= hi_idx && hi_idx < next) hi = cv[kFastCand + i];
              cum = next;
            }
            A.lo[(size_t)g * M + flist[a]] = lo;
            A.hi[(size_t)g * M + flist[a]] = hi;
          }
          __syncwarp();
        }
        __syncthreads();
        continue;
      }
      // Larger groups: per metric, histogram the median rank pair of every draw.
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
  if constexpr (kDeliver) {
    __syncthreads();   // the group's outputs (written by several threads) are complete
    deliver_groups(X, A, g);
  }
}

// Deliver the CTA's group (medians, lows, highs) to the gathered buffer of
// every receiving rank (all of them, or only X.root) with peer stores over
// NVLink; the last CTA of the launch raises this rank's arrival flag there.
// The barrier orders the CTA's stores before thread 0's acquire-release count
// (GPU scope: every counting CTA is on this GPU), and the last CTA releases
// them all with its system-scope flag stores.
__device__ __forceinline__ bool receives(const pm_peer_groups& X, int r) { return X.root < 0 || r == X.root; }

__device__ __noinline__ void deliver_groups(const pm_peer_groups& X, const BootArgs& A, int g) {
  const int M = A.n_metrics;
  for (int r = 0; r < X.n_ranks; ++r) {
    if (!receives(X, r)) continue;
    for (int i = threadIdx.x; i < 3 * M; i += blockDim.x) {
      const int k = i / M, m = i - k * M;
      const double* src = k == 0 ? A.medians : k == 1 ? A.lo : A.hi;
      X.out[r][(((size_t)X.rank * 3 + k) * X.per_rank + g) * M + m] = src[(size_t)g * M + m];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t prev;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(X.done) : "memory");
    if (prev + 1u == X.epoch * gridDim.x)
      for (int r = 0; r < X.n_ranks; ++r)
        if (receives(X, r))
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(X.flags[r] + X.rank), "r"(X.epoch) : "memory");
  }
}

// This rank owns no group: raise its arrival flag on every receiving rank at once.
__global__ void signal_groups_kernel(pm_peer_groups X) {
  if (threadIdx.x == 0)
    for (int r = 0; r < X.n_ranks; ++r)
      if (receives(X, r))
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(X.flags[r] + X.rank), "r"(X.epoch) : "memory");
}

// Raw index stream (diagnostic): out[r*n + j] for one seed, by one CTA.
__global__ void resample_indices_kernel(uint64_t seed, int n, int B, int32_t* out) {
  __shared__ uint32_t mt[2][kMtN];
  __shared__ uint32_t ring[kRing];
  if (threadIdx.x == 0) seed_state(mt[0], seed, ConstInit{});
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
// Generator constants uploaded per device, once: host threads calling on the
// same device take the lock; a device whose upload is done skips it.
static std::atomic<bool> g_constants_ready[64];
static std::mutex g_constants_lock;

int prepare_bootstrap_constants(int device) {
  if (device < 0 || device >= 64) return 1;
  if (g_constants_ready[device].load(std::memory_order_acquire)) return 0;
  std::lock_guard<std::mutex> guard(g_constants_lock);
  if (g_constants_ready[device].load(std::memory_order_relaxed)) return 0;
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
  g_constants_ready[device].store(true, std::memory_order_release);
  return 0;
}

size_t bootstrap_scratch_bytes(int n_groups, int max_members, int resamples, bool streamed) {
  return hist_area_bytes(n_groups) +
         (streamed || max_members > kHistMaxN ? (size_t)n_groups * resamples * max_members : 0);
}

// Shared memory the fold needs for M metrics and groups of up to mm members,
// against what one CTA may use on the current device: 0 if it fits, else the
// bytes needed (written to *available the bytes the device offers).
size_t bootstrap_smem_shortfall(int M, int mm, size_t* available) {
  const size_t dyn = BootSmem(M, mm, mm > kHistMaxN).total;
  // Both queries are answered once (per process, per device): they sit on
  // every bootstrap call's host path.
  static const size_t static_bytes = [] {
    cudaFuncAttributes attr{};
    const size_t b = cudaFuncGetAttributes(&attr, bootstrap_kernel<false>) == cudaSuccess ? attr.sharedSizeBytes : 0;
    cudaGetLastError();   // a failed query must not surface as a later launch error
    return b;
  }();
  static std::atomic<int> optin_of[kMaxDevices];
  int dev = 0, optin = 48 * 1024;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    optin = optin_of[dev].load(std::memory_order_relaxed);
    if (optin == 0) {
      optin = 48 * 1024;
      if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess)
        optin_of[dev].store(optin, std::memory_order_relaxed);
    }
  }
  cudaGetLastError();
  if (available) *available = (size_t)optin;
  return static_bytes + dyn <= (size_t)optin ? 0 : static_bytes + dyn;
}

int launch_bootstrap(const BootArgs& A, cudaStream_t stream, const pm_peer_groups* groups) {
  pm_peer_groups X{};
  if (groups) X = *groups;
  if (A.n_groups == 0) {
    if (X.n_ranks > 0) signal_groups_kernel<<<1, 32, 0, stream>>>(X);
    return 0;
  }
  const size_t smem = BootSmem(A.n_metrics, A.max_members, A.max_members > kHistMaxN).total;
  // The kernel's static shared memory, for the opt-in check.
  static size_t static_bytes = [] {
    cudaFuncAttributes attr{};
    return cudaFuncGetAttributes(&attr, bootstrap_kernel<false>) == cudaSuccess ? attr.sharedSizeBytes : size_t(48 * 1024);
  }();
  if (X.n_ranks > 0) {
    static std::atomic<int> limits[kMaxDevices];
    ensure_dynamic_smem(bootstrap_kernel<true>, static_bytes, smem, limits);
    bootstrap_kernel<true><<<A.n_groups, kBootThreads, smem, stream>>>(A, X);
  } else {
    static std::atomic<int> limits[kMaxDevices];
    ensure_dynamic_smem(bootstrap_kernel<false>, static_bytes, smem, limits);
    bootstrap_kernel<false><<<A.n_groups, kBootThreads, smem, stream>>>(A, X);
  }
  return 0;
}

int launch_bootstrap_prepare(const BootArgs& A, cudaStream_t stream) {
  if (A.n_groups == 0) return 0;
  bootstrap_prepare_kernel<<<A.n_groups, kPrepThreads, 0, stream>>>(A);
  return 0;
}

int launch_resample_indices(uint64_t seed, int n, int B, int32_t* out, cudaStream_t stream) {
  resample_indices_kernel<<<1, kBootThreads, 0, stream>>>(seed, n, B, out);
  return 0;
}

}  // namespace pm
