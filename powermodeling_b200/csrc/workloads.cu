// Workload kernels of the measured arms, sm_100a.
//
// Memory arms keep the reference's address sequences (gpu_bench.cu:326-406):
// thread t of L lanes starts at (t*stride) mod n and advances by
// (L*stride) mod n, so a per-thread sum or XOR is defined by the geometry and
// the fill alone and is checked against the CPU oracle.  Loads use the cache
// policy intrinsics (__ldca/__ldcg/__ldcs, i.e. ld.global.{ca,cg,cs}) rather
// than volatile asm, so the compiler keeps several loads in flight per thread;
// 16-byte vector modes move four words per access.
#include "workloads.cuh"

#include <cuda_fp16.h>
#include <string_view>

namespace pm {

__device__ __forceinline__ unsigned smid() {
  unsigned id;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(id));
  return id;
}

// Admit the block if its SM passes the filter; count admitted blocks per SM.
__device__ __forceinline__ bool admit(const Admission& a) {
  const unsigned id = smid();
  const bool ok = id < kSmSlots && (!a.filtered || a.mask[id]);
  if (ok && threadIdx.x == 0) atomicAdd(a.blocks_per_sm + id, 1ULL);
  return ok;
}

template <int P> __device__ __forceinline__ uint32_t load_word(const uint32_t* p) {
  if constexpr (P == RP_CA) return __ldca(p);
  else if constexpr (P == RP_CG) return __ldcg(p);
  else return __ldcs(p);
}
template <int P> __device__ __forceinline__ uint4 load_quad(const uint4* p) {
  if constexpr (P == RP_CA) return __ldca(p);
  else if constexpr (P == RP_CG) return __ldcg(p);
  else return __ldcs(p);
}

__device__ __forceinline__ uint64_t add_wrap(uint64_t a, uint64_t b, uint64_t n) {
  const uint64_t s = a + b;
  return s >= n ? s - n : s;
}

// ---------------------------------------------------------------------------
__global__ void fill_words_kernel(uint32_t* data, uint64_t n, uint64_t seed, int fill) {
  const uint64_t quads = n / 4;
  const uint64_t step = uint64_t(gridDim.x) * blockDim.x;
  uint4* q = reinterpret_cast<uint4*>(data);
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < quads; i += step) {
    const uint64_t w = 4 * i;
    if (fill == FILL_LCG) {
      const uint32_t x0 = lcg_word(w, seed), x1 = 1664525U * x0 + 1013904223U, x2 = 1664525U * x1 + 1013904223U;
      q[i] = make_uint4(x0, x1, x2, 1664525U * x2 + 1013904223U);
    } else {
      q[i] = make_uint4(random_word(w ^ seed), random_word((w + 1) ^ seed), random_word((w + 2) ^ seed),
                        random_word((w + 3) ^ seed));
    }
  }
  for (uint64_t w = 4 * quads + uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; w < n; w += step)
    data[w] = fill == FILL_LCG ? lcg_word(w, seed) : random_word(w ^ seed);
}

// fp16 operands: the reference's [-0.25, 0.25) grid (gpu_bench.cu:287-290) or
// uniform[-1, 1) on the same 16-bit lattice.
__global__ void fill_halves_kernel(unsigned short* data, uint64_t n, uint64_t seed, int uniform_pm1) {
  const uint64_t step = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += step) {
    const float v = uniform_pm1 ? (float(int(random_word(i ^ seed) & 65535U)) - 32768.0f) / 32768.0f
                                : (float(int(random_word(i ^ seed) & 65535U)) - 32768.0f) / 131072.0f;
    data[i] = __half_as_ushort(__float2half(v));
  }
}

// ---------------------------------------------------------------------------
// Scalar single-stream read: sum32 of `iterations` words per thread.
template <int P, bool L1, bool Narrow>
__global__ void read_scalar_kernel(const uint32_t* in, uint32_t* sink, uint64_t total, uint64_t slice, uint64_t stride,
                                   uint64_t iterations, Admission adm) {
  if (!admit(adm)) return;
  const uint64_t n = L1 ? slice : total;
  const uint64_t lanes = L1 ? blockDim.x : uint64_t(gridDim.x) * blockDim.x;
  const uint64_t tid = L1 ? threadIdx.x : uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint32_t* base = L1 ? in + uint64_t(blockIdx.x) * slice : in;
  uint32_t sum = 0;
  if constexpr (Narrow) {
    uint32_t pos = uint32_t((tid * stride) % n);
    const uint32_t adv = uint32_t((lanes * stride) % n);
    const uint32_t boundary = uint32_t(n) - adv;
    const uint32_t iters = uint32_t(iterations);
#pragma unroll 8
    for (uint32_t i = 0; i < iters; ++i) {
      sum += load_word<P>(base + pos);
      pos = pos >= boundary ? pos - boundary : pos + adv;
    }
  } else {
    uint64_t pos = (tid * stride) % n;
    const uint64_t adv = (lanes * stride) % n;
#pragma unroll 8
    for (uint64_t i = 0; i < iterations; ++i) {
      sum += load_word<P>(base + pos);
      pos = add_wrap(pos, adv, n);
    }
  }
  sink[uint64_t(blockIdx.x) * blockDim.x + threadIdx.x] = sum;
}

// 16-byte read: sum32 of every word of `iterations` quads per thread, quads
// addressed like words of the scalar read (stride in quads).
template <int P>
__global__ void read_vector_kernel(const uint4* in, uint32_t* sink, uint64_t quads, uint64_t stride, uint64_t iterations,
                                   Admission adm) {
  if (!admit(adm)) return;
  const uint64_t lanes = uint64_t(gridDim.x) * blockDim.x;
  const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  uint64_t pos = (tid * stride) % quads;
  const uint64_t adv = (lanes * stride) % quads;
  uint32_t sum = 0;
#pragma unroll 4
  for (uint64_t i = 0; i < iterations; ++i) {
    const uint4 v = load_quad<P>(in + pos);
    sum += v.x + v.y + v.z + v.w;
    pos = add_wrap(pos, adv, quads);
  }
  sink[tid] = sum;
}

// Four-stream write (Copy=false) or copy (Copy=true), gpu_bench.cu:359-406 semantics.
template <bool Copy>
__global__ void write_copy_scalar_kernel(const uint32_t* in, uint32_t* out, uint32_t* sink, uint64_t n, uint64_t stride,
                                         uint64_t iterations, Admission adm) {
  if (!admit(adm)) return;
  const uint64_t lanes = uint64_t(gridDim.x) * blockDim.x;
  const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  uint64_t base = (tid * stride) % n;
  const uint64_t d1 = (lanes * stride) % n, d2 = (lanes * 2 * stride) % n, d3 = (lanes * 3 * stride) % n;
  const uint64_t adv = (lanes * 4 * stride) % n;
  uint32_t a = random_word(tid), b = a ^ 0x7f4a7c15U, c = a ^ 0xbf58476dU, d = a ^ 0x94d049bbU;
  for (uint64_t i = 0; i < iterations; ++i) {
    const uint64_t j0 = base, j1 = add_wrap(base, d1, n), j2 = add_wrap(base, d2, n), j3 = add_wrap(base, d3, n);
    if constexpr (Copy) {
      const uint32_t x0 = __ldcg(in + j0), x1 = __ldcg(in + j1), x2 = __ldcg(in + j2), x3 = __ldcg(in + j3);
      __stcg(out + j0, x0); __stcg(out + j1, x1); __stcg(out + j2, x2); __stcg(out + j3, x3);
      a ^= x0; b ^= x1; c ^= x2; d ^= x3;
    } else {
      a = a * 1664525U + 1013904223U; b ^= a + uint32_t(i);
      c = c * 22695477U + 1U; d ^= c + uint32_t(tid);
      __stcg(out + j0, a); __stcg(out + j1, b); __stcg(out + j2, c); __stcg(out + j3, d);
    }
    base = add_wrap(base, adv, n);
  }
  sink[tid] = a ^ b ^ c ^ d;
}

// 16-byte copy: quads move with streaming loads and stores; sink = XOR of the words copied.
__global__ void copy_vector_kernel(const uint4* in, uint4* out, uint32_t* sink, uint64_t quads, uint64_t stride,
                                   uint64_t iterations, Admission adm) {
  if (!admit(adm)) return;
  const uint64_t lanes = uint64_t(gridDim.x) * blockDim.x;
  const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  uint64_t pos = (tid * stride) % quads;
  const uint64_t adv = (lanes * stride) % quads;
  uint32_t x = 0;
#pragma unroll 4
  for (uint64_t i = 0; i < iterations; ++i) {
    const uint4 v = __ldcs(in + pos);
    __stcs(out + pos, v);
    x ^= v.x ^ v.y ^ v.z ^ v.w;
    pos = add_wrap(pos, adv, quads);
  }
  sink[tid] = x;
}

// Integer issue loop, the paired active reference (gpu_bench.cu:408-418 arithmetic).
__global__ void control_kernel(uint32_t* sink, uint64_t iterations, Admission adm) {
  if (!admit(adm)) return;
  const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t a = random_word(tid), b = a + 1U, c = a + 2U, d = a + 3U;
  for (uint64_t i = 0; i < iterations; ++i) {
    asm volatile("add.u32 %0, %0, %4;\n\txor.b32 %1, %1, %0;\n\tadd.u32 %2, %2, %1;\n\txor.b32 %3, %3, %2;"
                 : "+r"(a), "+r"(b), "+r"(c), "+r"(d) : "r"(uint32_t(i)));
  }
  sink[tid] = a ^ b ^ c ^ d;
}

// Dependent chase over 32-bit word links, one lane per block (gpu_bench.cu:457-473 semantics).
__global__ void chase_words_kernel(const uint32_t* links, uint32_t* sink, uint64_t words, uint64_t iterations,
                                   uint64_t nonce, Admission adm, unsigned long long* cycles, unsigned long long* loads) {
  if (!admit(adm) || threadIdx.x != 0) return;
  uint32_t index = uint32_t(random_word(nonce ^ (uint64_t(blockIdx.x) << 32)) % words);
  const unsigned long long begin = clock64();
  for (uint64_t i = 0; i < iterations; ++i) index = __ldcg(links + index);
  const unsigned long long elapsed = clock64() - begin;
  sink[uint64_t(blockIdx.x) * blockDim.x] = index;
  const unsigned id = smid();
  atomicAdd(cycles + id, elapsed);
  atomicAdd(loads + id, (unsigned long long)iterations);
}

// Dependent chase over 64-bit node indices on 128-byte lines: node k's link is
// the first word of line k.  One chain per block (lane 0 of a one-warp block).
__global__ void chase_lines_kernel(const uint64_t* lines, uint64_t* terminal, uint64_t nodes, uint64_t iterations,
                                   uint64_t nonce, Admission adm, unsigned long long* cycles, unsigned long long* loads) {
  if (!admit(adm) || threadIdx.x != 0) return;
  uint64_t index = random_word(nonce ^ (uint64_t(blockIdx.x) << 32)) % nodes;
  const unsigned long long begin = clock64();
  for (uint64_t i = 0; i < iterations; ++i) index = __ldcg(lines + index * 16);
  const unsigned long long elapsed = clock64() - begin;
  terminal[blockIdx.x] = index;
  const unsigned id = smid();
  atomicAdd(cycles + id, elapsed);
  atomicAdd(loads + id, (unsigned long long)iterations);
}

// ---------------------------------------------------------------------------
// Register SFU recurrence (sfu.cuh:43-105 semantics): y = MUFU(x);
// x = ((bits(y) ^ iteration) & 0x7fffff) | 0x3f000000; FNV-1a hash of the chains.
template <int Op, bool Control>
__device__ __forceinline__ uint32_t sfu_step(float x) {
  float y;
  if constexpr (Control) {
    uint32_t r;
    asm volatile("mov.b32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
  } else if constexpr (Op == SFU_EX2) {
    asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  } else if constexpr (Op == SFU_TANH) {
    asm volatile("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  } else if constexpr (Op == SFU_RSQRT) {
    asm volatile("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  } else if constexpr (Op == SFU_RCP) {
    asm volatile("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  } else if constexpr (Op == SFU_LG2) {
    asm volatile("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  } else {
    asm volatile("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  }
  return __float_as_uint(y);
}

template <int Op, bool Control, int Chains>
__global__ void sfu_kernel(uint32_t* sink, uint64_t lanes, uint64_t iterations, uint64_t seed, int input) {
  const uint64_t step = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t lane = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; lane < lanes; lane += step) {
    float state[Chains];
#pragma unroll
    for (int c = 0; c < Chains; ++c)
      state[c] = __uint_as_float(input == SFU_INPUT_UNIFORM_0P5_2 ? sfu_uniform_bits(lane, seed, c)
                                                                  : sfu_initial_bits(lane, seed, c));
#pragma unroll 1
    for (uint64_t it = 0; it < iterations; ++it) {
#pragma unroll
      for (int c = 0; c < Chains; ++c) {
        const uint32_t r = sfu_step<Op, Control>(state[c]);
        state[c] = __uint_as_float(((r ^ uint32_t(it)) & 0x007fffffU) | 0x3f000000U);
      }
    }
    uint32_t h = 2166136261U, x = 0;
#pragma unroll
    for (int c = 0; c < Chains; ++c) {
      h = (h ^ __float_as_uint(state[c])) * 16777619U;
      x ^= __float_as_uint(state[c]);
    }
    sink[lane] = input == SFU_INPUT_UNIFORM_0P5_2 ? x : h;
  }
}

// Eight one-step samples (x, MUFU(x)) for the CPU double-precision check (sfu.cuh:107-117).
template <int Op>
__global__ void sfu_check_kernel(uint32_t* sample, uint64_t lanes, uint64_t seed, int chains, int input) {
  const unsigned k = threadIdx.x;
  if (k >= 8) return;
  const uint64_t lane = uint64_t(k) * (lanes - 1) / 7;
  const int chain = int(k % unsigned(chains));
  const uint32_t bits = input == SFU_INPUT_UNIFORM_0P5_2 ? sfu_uniform_bits(lane, seed, chain)
                                                         : sfu_initial_bits(lane, seed, chain);
  sample[2 * k] = bits;
  sample[2 * k + 1] = sfu_step<Op, false>(__uint_as_float(bits));
}

// ---------------------------------------------------------------------------
static int fill_grid(uint64_t n, int sms) {
  const uint64_t want = (n / 4 + 255) / 256;
  const uint64_t cap = uint64_t(sms > 0 ? sms : 148) * 16;
  return int(want < 1 ? 1 : (want > cap ? cap : want));
}

cudaError_t launch_fill_words(uint32_t* data, uint64_t n, uint64_t seed, int sms, cudaStream_t s, int fill) {
  fill_words_kernel<<<fill_grid(n, sms), 256, 0, s>>>(data, n, seed, fill);
  return cudaGetLastError();
}

cudaError_t launch_fill_halves(void* data, uint64_t n, uint64_t seed, int uniform_pm1, int sms, cudaStream_t s) {
  fill_halves_kernel<<<fill_grid(4 * n, sms), 256, 0, s>>>(static_cast<unsigned short*>(data), n, seed, uniform_pm1);
  return cudaGetLastError();
}

cudaError_t launch_read_scalar(int policy, bool l1, const uint32_t* in, uint32_t* sink, uint64_t words, uint64_t slice,
                               uint64_t stride, uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s) {
  const uint64_t region = l1 ? slice : words;
  const bool narrow = region <= 0xffffffffULL && iterations <= 0xffffffffULL;
#define PM_READ(P, L, NR) read_scalar_kernel<P, L, NR><<<blocks, threads, 0, s>>>(in, sink, words, slice, stride, iterations, adm)
  if (l1) { if (narrow) PM_READ(RP_CA, true, true); else PM_READ(RP_CA, true, false); }
  else if (policy == RP_CA) { if (narrow) PM_READ(RP_CA, false, true); else PM_READ(RP_CA, false, false); }
  else if (policy == RP_CS) { if (narrow) PM_READ(RP_CS, false, true); else PM_READ(RP_CS, false, false); }
  else { if (narrow) PM_READ(RP_CG, false, true); else PM_READ(RP_CG, false, false); }
#undef PM_READ
  return cudaGetLastError();
}

cudaError_t launch_read_vector(int policy, const uint32_t* in, uint32_t* sink, uint64_t quads, uint64_t stride,
                               uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s) {
  const uint4* q = reinterpret_cast<const uint4*>(in);
  if (policy == RP_CA) read_vector_kernel<RP_CA><<<blocks, threads, 0, s>>>(q, sink, quads, stride, iterations, adm);
  else if (policy == RP_CS) read_vector_kernel<RP_CS><<<blocks, threads, 0, s>>>(q, sink, quads, stride, iterations, adm);
  else read_vector_kernel<RP_CG><<<blocks, threads, 0, s>>>(q, sink, quads, stride, iterations, adm);
  return cudaGetLastError();
}

cudaError_t launch_write_copy_scalar(bool copy, const uint32_t* in, uint32_t* out, uint32_t* sink, uint64_t words,
                                     uint64_t stride, uint64_t iterations, int blocks, int threads, Admission adm,
                                     cudaStream_t s) {
  if (copy) write_copy_scalar_kernel<true><<<blocks, threads, 0, s>>>(in, out, sink, words, stride, iterations, adm);
  else write_copy_scalar_kernel<false><<<blocks, threads, 0, s>>>(in, out, sink, words, stride, iterations, adm);
  return cudaGetLastError();
}

cudaError_t launch_copy_vector(const uint32_t* in, uint32_t* out, uint32_t* sink, uint64_t quads, uint64_t stride,
                               uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s) {
  copy_vector_kernel<<<blocks, threads, 0, s>>>(reinterpret_cast<const uint4*>(in), reinterpret_cast<uint4*>(out), sink,
                                                quads, stride, iterations, adm);
  return cudaGetLastError();
}

cudaError_t launch_control(uint32_t* sink, uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s) {
  control_kernel<<<blocks, threads, 0, s>>>(sink, iterations, adm);
  return cudaGetLastError();
}

cudaError_t launch_chase_words(const uint32_t* links, uint32_t* sink, uint64_t words, uint64_t iterations, uint64_t nonce,
                               int blocks, int threads, Admission adm, unsigned long long* cycles,
                               unsigned long long* loads, cudaStream_t s) {
  chase_words_kernel<<<blocks, threads, 0, s>>>(links, sink, words, iterations, nonce, adm, cycles, loads);
  return cudaGetLastError();
}

cudaError_t launch_chase_lines(const uint64_t* lines, uint64_t* terminal, uint64_t nodes, uint64_t iterations,
                               uint64_t nonce, int blocks, int threads, Admission adm, unsigned long long* cycles,
                               unsigned long long* loads, cudaStream_t s) {
  chase_lines_kernel<<<blocks, threads, 0, s>>>(lines, terminal, nodes, iterations, nonce, adm, cycles, loads);
  return cudaGetLastError();
}

template <int Op, bool Control>
static void sfu_dispatch_chains(int chains, uint32_t* sink, uint64_t lanes, uint64_t it, uint64_t seed, int b, int t,
                                cudaStream_t s, int input) {
  if (chains == 1) sfu_kernel<Op, Control, 1><<<b, t, 0, s>>>(sink, lanes, it, seed, input);
  else if (chains == 4) sfu_kernel<Op, Control, 4><<<b, t, 0, s>>>(sink, lanes, it, seed, input);
  else sfu_kernel<Op, Control, 8><<<b, t, 0, s>>>(sink, lanes, it, seed, input);
}

cudaError_t launch_sfu(int op, bool control, int chains, uint32_t* sink, uint64_t lanes, uint64_t iterations,
                       uint64_t seed, int blocks, int threads, cudaStream_t s, int input) {
#define PM_SFU(OP, CTRL) sfu_dispatch_chains<OP, CTRL>(chains, sink, lanes, iterations, seed, blocks, threads, s, input)
  if (control) { PM_SFU(SFU_EX2, true); return cudaGetLastError(); }
  switch (op) {
    case SFU_EX2: PM_SFU(SFU_EX2, false); break;
    case SFU_TANH: PM_SFU(SFU_TANH, false); break;
    case SFU_RSQRT: PM_SFU(SFU_RSQRT, false); break;
    case SFU_RCP: PM_SFU(SFU_RCP, false); break;
    case SFU_LG2: PM_SFU(SFU_LG2, false); break;
    default: PM_SFU(SFU_SQRT, false); break;
  }
#undef PM_SFU
  return cudaGetLastError();
}

cudaError_t launch_sfu_check(int op, uint32_t* sample, uint64_t lanes, uint64_t seed, int chains, cudaStream_t s,
                             int input) {
  switch (op) {
    case SFU_EX2: sfu_check_kernel<SFU_EX2><<<1, 32, 0, s>>>(sample, lanes, seed, chains, input); break;
    case SFU_TANH: sfu_check_kernel<SFU_TANH><<<1, 32, 0, s>>>(sample, lanes, seed, chains, input); break;
    case SFU_RSQRT: sfu_check_kernel<SFU_RSQRT><<<1, 32, 0, s>>>(sample, lanes, seed, chains, input); break;
    case SFU_RCP: sfu_check_kernel<SFU_RCP><<<1, 32, 0, s>>>(sample, lanes, seed, chains, input); break;
    case SFU_LG2: sfu_check_kernel<SFU_LG2><<<1, 32, 0, s>>>(sample, lanes, seed, chains, input); break;
    default: sfu_check_kernel<SFU_SQRT><<<1, 32, 0, s>>>(sample, lanes, seed, chains, input); break;
  }
  return cudaGetLastError();
}

template <int Op, bool Control>
static cudaError_t sfu_attr_chains(int chains, cudaFuncAttributes* a) {
  if (chains == 1) return cudaFuncGetAttributes(a, sfu_kernel<Op, Control, 1>);
  if (chains == 4) return cudaFuncGetAttributes(a, sfu_kernel<Op, Control, 4>);
  return cudaFuncGetAttributes(a, sfu_kernel<Op, Control, 8>);
}

cudaError_t sfu_attributes(int op, bool control, int chains, cudaFuncAttributes* attr) {
  if (control) return sfu_attr_chains<SFU_EX2, true>(chains, attr);
  switch (op) {
    case SFU_EX2: return sfu_attr_chains<SFU_EX2, false>(chains, attr);
    case SFU_TANH: return sfu_attr_chains<SFU_TANH, false>(chains, attr);
    case SFU_RSQRT: return sfu_attr_chains<SFU_RSQRT, false>(chains, attr);
    case SFU_RCP: return sfu_attr_chains<SFU_RCP, false>(chains, attr);
    case SFU_LG2: return sfu_attr_chains<SFU_LG2, false>(chains, attr);
    default: return sfu_attr_chains<SFU_SQRT, false>(chains, attr);
  }
}

template <int Op, bool Control>
static const void* sfu_handle_chains(int chains) {
  if (chains == 1) return (const void*)sfu_kernel<Op, Control, 1>;
  if (chains == 4) return (const void*)sfu_kernel<Op, Control, 4>;
  return (const void*)sfu_kernel<Op, Control, 8>;
}

const void* sfu_kernel_handle(int op, bool control, int chains) {
  if (control) return sfu_handle_chains<SFU_EX2, true>(chains);
  switch (op) {
    case SFU_EX2: return sfu_handle_chains<SFU_EX2, false>(chains);
    case SFU_TANH: return sfu_handle_chains<SFU_TANH, false>(chains);
    case SFU_RSQRT: return sfu_handle_chains<SFU_RSQRT, false>(chains);
    case SFU_RCP: return sfu_handle_chains<SFU_RCP, false>(chains);
    case SFU_LG2: return sfu_handle_chains<SFU_LG2, false>(chains);
    default: return sfu_handle_chains<SFU_SQRT, false>(chains);
  }
}

// Kernel handles for resource queries (cudaFuncGetAttributes / occupancy).
const void* kernel_symbol(const char* name, int a, int b, int c) {
  (void)c;
  const std::string_view n(name);
  if (n == "read_scalar") {
    if (a == 3) return b ? (const void*)read_scalar_kernel<RP_CA, true, true> : (const void*)read_scalar_kernel<RP_CA, true, false>;
    if (a == RP_CA) return b ? (const void*)read_scalar_kernel<RP_CA, false, true> : (const void*)read_scalar_kernel<RP_CA, false, false>;
    if (a == RP_CS) return b ? (const void*)read_scalar_kernel<RP_CS, false, true> : (const void*)read_scalar_kernel<RP_CS, false, false>;
    return b ? (const void*)read_scalar_kernel<RP_CG, false, true> : (const void*)read_scalar_kernel<RP_CG, false, false>;
  }
  if (n == "read_vector") return a == RP_CA ? (const void*)read_vector_kernel<RP_CA> : a == RP_CS ? (const void*)read_vector_kernel<RP_CS> : (const void*)read_vector_kernel<RP_CG>;
  if (n == "write_scalar") return (const void*)write_copy_scalar_kernel<false>;
  if (n == "copy_scalar") return (const void*)write_copy_scalar_kernel<true>;
  if (n == "copy_vector") return (const void*)copy_vector_kernel;
  if (n == "control") return (const void*)control_kernel;
  if (n == "chase_words") return (const void*)chase_words_kernel;
  if (n == "chase_lines") return (const void*)chase_lines_kernel;
  return nullptr;
}

}  // namespace pm
