// Oracle (test infrastructure only): CPU restatement of the deterministic
// workload bookkeeping of the reference's powerbench (cuda/gpu_bench.cu):
// the word fill random_word (277-282), per-thread read sums over the
// stride-wrapped address sequence (326-357, CPU check 937-973), the
// four-stream write/copy sinks (359-406), the integer issue loop (408-418),
// the full-cycle chase permutation (722-731) and its walk (457-473), the SFU
// initial operands (sfu.cuh:73-75) and the sampled sink hash (984-996).
// It also states the 16-byte access variants of this library.  Built by
// oracle/build_oracle.py into liboracle_words.so and called from the tests.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <random>
#include <vector>

extern "C" {

uint32_t oracle_random_word(uint64_t x) {
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return uint32_t(x ^ (x >> 31));
}

uint64_t oracle_sink_hash(const uint32_t* words, uint64_t n) {
  uint64_t h = 0;
  for (uint64_t i = 0; i < n; ++i) h = h * 1315423911ULL + words[i];
  return h;
}

uint64_t oracle_u64_hash(const uint64_t* words, uint64_t n) {
  uint64_t h = 0;
  for (uint64_t i = 0; i < n; ++i) h = h * 1315423911ULL + words[i];
  return h;
}

// Sum32 of every thread's reads.  unit = 1 (scalar word) or 4 (16-byte quad);
// for L1 (slice > 0) thread ids restart per block and each block reads its slice.
// As oracle_read_sums over an explicit payload (buffer word i = payload[i]),
// for the fills other than random_word.
void oracle_read_sums_of(const uint32_t* payload, uint64_t words, uint64_t offset_words, uint64_t blocks,
                         uint64_t threads, uint64_t stride, uint64_t iterations, uint64_t slice, uint64_t unit,
                         uint32_t* out, uint64_t count) {
  const bool l1 = slice > 0;
  const uint64_t lanes = blocks * threads;
  const uint64_t region = (l1 ? slice : words) / unit;
  const uint64_t region_lanes = l1 ? threads : lanes;
  const uint64_t advance = (region_lanes * stride) % region;
  for (uint64_t g = 0; g < count && g < lanes; ++g) {
    const uint64_t block = g / threads, tid = l1 ? g % threads : g;
    uint64_t pos = (tid * stride) % region;
    uint32_t sum = 0;
    for (uint64_t k = 0; k < iterations; ++k) {
      for (uint64_t w = 0; w < unit; ++w) sum += payload[offset_words + (l1 ? block * slice : 0) + pos * unit + w];
      pos = (pos + advance) % region;
    }
    out[g] = sum;
  }
}

void oracle_read_sums(uint64_t words, uint64_t offset_words, uint64_t seed, uint64_t blocks, uint64_t threads,
                      uint64_t stride, uint64_t iterations, uint64_t slice, uint64_t unit, uint32_t* out, uint64_t count) {
  const bool l1 = slice > 0;
  const uint64_t lanes = blocks * threads;
  const uint64_t region = (l1 ? slice : words) / unit;
  const uint64_t region_lanes = l1 ? threads : lanes;
  const uint64_t advance = (region_lanes * stride) % region;
  for (uint64_t g = 0; g < count && g < lanes; ++g) {
    const uint64_t block = g / threads, tid = l1 ? g % threads : g;
    uint64_t pos = (tid * stride) % region;
    uint32_t sum = 0;
    for (uint64_t k = 0; k < iterations; ++k) {
      for (uint64_t w = 0; w < unit; ++w)
        sum += oracle_random_word((offset_words + (l1 ? block * slice : 0) + pos * unit + w) ^ seed);
      pos = (pos + advance) % region;
    }
    out[g] = sum;
  }
}

// Sink of the four-stream write (copy = 0) or copy (copy = 1) thread g.
void oracle_write_copy_sinks(uint64_t words, uint64_t offset_words, uint64_t seed, uint64_t blocks, uint64_t threads,
                             uint64_t stride, uint64_t iterations, int copy, uint32_t* out, uint64_t count) {
  const uint64_t n = words, lanes = blocks * threads;
  const uint64_t d1 = (lanes * stride) % n, d2 = (lanes * 2 * stride) % n, d3 = (lanes * 3 * stride) % n;
  const uint64_t adv = (lanes * 4 * stride) % n;
  auto wrap = [n](uint64_t a, uint64_t b) { const uint64_t s = a + b; return s >= n ? s - n : s; };
  for (uint64_t tid = 0; tid < count && tid < lanes; ++tid) {
    uint64_t base = (tid * stride) % n;
    uint32_t a = oracle_random_word(tid), b = a ^ 0x7f4a7c15U, c = a ^ 0xbf58476dU, d = a ^ 0x94d049bbU;
    for (uint64_t i = 0; i < iterations; ++i) {
      const uint64_t j[4] = {base, wrap(base, d1), wrap(base, d2), wrap(base, d3)};
      if (copy) {
        a ^= oracle_random_word((offset_words + j[0]) ^ seed); b ^= oracle_random_word((offset_words + j[1]) ^ seed);
        c ^= oracle_random_word((offset_words + j[2]) ^ seed); d ^= oracle_random_word((offset_words + j[3]) ^ seed);
      } else {
        a = a * 1664525U + 1013904223U; b ^= a + uint32_t(i);
        c = c * 22695477U + 1U; d ^= c + uint32_t(tid);
      }
      base = wrap(base, adv);
    }
    out[tid] = a ^ b ^ c ^ d;
  }
}

// XOR of the words a 16-byte copy thread moves.
void oracle_copy_vector_sinks(uint64_t quads, uint64_t offset_words, uint64_t seed, uint64_t blocks, uint64_t threads,
                              uint64_t stride, uint64_t iterations, uint32_t* out, uint64_t count) {
  const uint64_t lanes = blocks * threads, adv = (lanes * stride) % quads;
  for (uint64_t tid = 0; tid < count && tid < lanes; ++tid) {
    uint64_t pos = (tid * stride) % quads;
    uint32_t x = 0;
    for (uint64_t i = 0; i < iterations; ++i) {
      for (uint64_t w = 0; w < 4; ++w) x ^= oracle_random_word((offset_words + pos * 4 + w) ^ seed);
      pos = (pos + adv) % quads;
    }
    out[tid] = x;
  }
}

void oracle_control_sinks(uint64_t iterations, uint32_t* out, uint64_t count) {
  for (uint64_t tid = 0; tid < count; ++tid) {
    uint32_t a = oracle_random_word(tid), b = a + 1U, c = a + 2U, d = a + 3U;
    for (uint64_t i = 0; i < iterations; ++i) { a += uint32_t(i); b ^= a; c += b; d ^= c; }
    out[tid] = a ^ b ^ c ^ d;
  }
}

// Next-node table of the full random cycle: next[order[k]] = order[k + 1].
void oracle_chase_links(uint64_t nodes, uint64_t seed, uint32_t* next) {
  std::vector<uint32_t> order(nodes);
  std::iota(order.begin(), order.end(), 0U);
  std::mt19937_64 gen(seed);
  std::shuffle(order.begin(), order.end(), gen);
  for (uint64_t k = 0; k < nodes; ++k) next[order[k]] = order[(k + 1) % nodes];
}

// Terminal node of block b's chain after `iterations` dependent loads.
uint64_t oracle_chase_terminal(const uint32_t* next, uint64_t nodes, uint64_t iterations, uint64_t nonce, uint64_t block) {
  uint64_t index = oracle_random_word(nonce ^ (block << 32)) % nodes;
  for (uint64_t i = 0; i < iterations; ++i) index = next[index];
  return index;
}

uint32_t oracle_sfu_initial_bits(uint64_t lane, uint64_t seed, int chain) {
  return (oracle_random_word(lane ^ seed ^ (uint64_t(chain + 1) * 0x9e3779b97f4a7c15ULL)) & 0x007fffffU) | 0x3f000000U;
}

// Seeded uint32 LCG fill (the memory arms' extra mode): x_0 = low 32 bits of the
// seed, x_{i+1} = 1664525 x_i + 1013904223 mod 2^32, stepped one word at a time
// (the product reaches word i by squaring the step; the two must agree).
void oracle_lcg_words(uint64_t n, uint64_t seed, uint32_t* out) {
  uint32_t x = uint32_t(seed);
  for (uint64_t i = 0; i < n; ++i) {
    out[i] = x;
    x = 1664525U * x + 1013904223U;
  }
}

// The SFU arm's extra-mode operand: uniform [0.5, 2.0) from the lane hash,
// 0.5 + 1.5 m / 2^24 for the hash's top 24 bits m, each float operation rounded.
uint32_t oracle_sfu_uniform_bits(uint64_t lane, uint64_t seed, int chain) {
  const uint32_t m = oracle_random_word(lane ^ seed ^ (uint64_t(chain + 1) * 0x9e3779b97f4a7c15ULL)) >> 8;
  volatile float scaled = float(m) * (1.5f / 16777216.0f);
  const float x = scaled + 0.5f;
  uint32_t bits;
  memcpy(&bits, &x, 4);
  return bits;
}

}  // extern "C"
