// Complete FP32 nonlinear functions of the powerbench exp|tanh|silu|rmsnorm|softmax
// workloads (the reference's cuda/nonlinear.cuh, opt-in with --nonlinear-mode streaming).
//
// Semantics kept from the reference: the deterministic input and gamma fill
// (nonlinear.cuh:5-14), one output per input element per repeat, every repeat
// reloading the fixed input from global memory (nonlinear.cuh:23-38, 59-89),
// expf / tanhf / x/(1+expf(-x)) for the pointwise functions, stable
// max-subtracted softmax, and RMSNorm y = x * rsqrtf(mean(x^2) + 1e-5) * gamma.
// The user's grid and block size are the experiment's launch geometry; what
// a CTA does inside it is B200-specific:
//  * pointwise: grid-stride over 16-byte quads, four independent quads in
//    flight per thread (64 bytes), ld/st.global.cg, a scalar tail of n mod 4;
//  * row-wise, grid-stride grids with at least one row per warp and rows of
//    at most 1024 floats (a multiple of 4): one warp per row, the row held in
//    registers (up to 8 quads per lane), warp-shuffle reductions, no shared
//    memory or barriers; every input byte crosses HBM once;
//  * row-wise, one CTA per row (as the auto grid launches) with rows of at most
//    16 x threads floats (a multiple of 4): the row in registers (up to 4
//    quads per thread), two block reductions over float4-read partials;
//  * row-wise otherwise (wider rows, widths not a multiple of 4): each
//    thread owns the same quads of a row in every pass; the row is staged in
//    shared memory once (rows up to kRowStageFloats floats), so HBM sees each
//    input byte once instead of two (RMSNorm) or three (softmax) times;
//    softmax keeps exp(x - max) in the staged row instead of re-evaluating
//    it; reductions are warp shuffles plus one cross-warp step in a fixed
//    order, alternating two buffers so one barrier per reduction suffices.
//    Wider rows re-read global memory in each pass.
// This file is compiled with contraction (fmad) enabled like the reference, so
// the pointwise outputs equal the reference kernel's bit for bit.
#include "workloads.cuh"

#include <atomic>
#include <cstdint>

#include "pm_capi.h"
#include "pmb200.h"

namespace pm {

namespace {

constexpr float kRmsEpsilon = 1e-5f;
constexpr int kMaxWarps = 32;
constexpr int kRowStageFloats = 40960;             // 160 KiB of staged row per CTA

__device__ __forceinline__ uint4 ld_cg4(const float* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_cg4(float* p, uint4 v) {
  asm volatile("st.global.cg.v4.u32 [%0], {%1,%2,%3,%4};" :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
}
__device__ __forceinline__ float ld_cg1(const float* p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return __uint_as_float(v);
}
__device__ __forceinline__ void st_cg1(float* p, float x) {
  asm volatile("st.global.cg.u32 [%0], %1;" :: "l"(p), "r"(__float_as_uint(x)));
}

// ---------------------------------------------------------------- fill
__global__ void nonlinear_fill_kernel(float* data, uint64_t n, uint64_t seed, float shift, int gamma) {
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t bits = random_word(i ^ seed) & 65535U;
    data[i] = gamma ? 0.75f + float(bits) / 131072.0f : float(int(bits) - 32768) / 8192.0f + shift;
  }
}

// ---------------------------------------------------------------- pointwise
template <int F> __device__ __forceinline__ float pointwise(float x) {
  if constexpr (F == NL_EXP) return expf(x);
  else if constexpr (F == NL_TANH) return tanhf(x);
  else return x / (1.0f + expf(-x));
}
template <int F> __device__ __forceinline__ uint4 pointwise4(uint4 v) {
  return make_uint4(__float_as_uint(pointwise<F>(__uint_as_float(v.x))), __float_as_uint(pointwise<F>(__uint_as_float(v.y))),
                    __float_as_uint(pointwise<F>(__uint_as_float(v.z))), __float_as_uint(pointwise<F>(__uint_as_float(v.w))));
}

template <int F>
__global__ void __launch_bounds__(1024) pointwise_stream_kernel(const float* in, float* out, uint64_t n,
                                                                uint64_t iterations) {
  const uint64_t quads = n >> 2, tail = n & 3;
  const uint64_t first = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t step = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t r = 0; r < iterations; ++r) {
    uint64_t q = first;
    for (; q + 3 * step < quads; q += 4 * step) {
      const uint4 a = ld_cg4(in + 4 * q), b = ld_cg4(in + 4 * (q + step));
      const uint4 c = ld_cg4(in + 4 * (q + 2 * step)), d = ld_cg4(in + 4 * (q + 3 * step));
      st_cg4(out + 4 * q, pointwise4<F>(a));
      st_cg4(out + 4 * (q + step), pointwise4<F>(b));
      st_cg4(out + 4 * (q + 2 * step), pointwise4<F>(c));
      st_cg4(out + 4 * (q + 3 * step), pointwise4<F>(d));
    }
    for (; q < quads; q += step) st_cg4(out + 4 * q, pointwise4<F>(ld_cg4(in + 4 * q)));
    if (first < tail) {
      const uint64_t i = 4 * quads + first;
      st_cg1(out + i, pointwise<F>(ld_cg1(in + i)));
    }
  }
}

// ---------------------------------------------------------------- row-wise
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// CTA-wide reduction; every thread returns the same value.  Consecutive calls
// must alternate `red` between two buffers: a thread writes buffer X at
// reduction j + 2 only after the barrier of reduction j + 1, by which time
// every thread has read reduction j's partials.
template <bool Max>
__device__ __forceinline__ float cta_reduce(float v, float* red) {
  v = Max ? warp_max(v) : warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  float r = red[0];
  for (int w = 1; w < warps; ++w) r = Max ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

// V floats per group: 4 (row width a multiple of 4: 16-byte aligned rows) or 1.
template <int V> struct alignas(4 * V) Group { float v[V]; };

template <int V> __device__ __forceinline__ Group<V> load_group(const float* p) {
  Group<V> g;
  if constexpr (V == 4) {
    const uint4 q = ld_cg4(p);
    g.v[0] = __uint_as_float(q.x); g.v[1] = __uint_as_float(q.y); g.v[2] = __uint_as_float(q.z); g.v[3] = __uint_as_float(q.w);
  } else {
    g.v[0] = ld_cg1(p);
  }
  return g;
}
template <int V> __device__ __forceinline__ void store_group(float* p, const Group<V>& g) {
  if constexpr (V == 4)
    st_cg4(p, make_uint4(__float_as_uint(g.v[0]), __float_as_uint(g.v[1]), __float_as_uint(g.v[2]), __float_as_uint(g.v[3])));
  else
    st_cg1(p, g.v[0]);
}
template <int V> __device__ __forceinline__ Group<V> gamma_group(const float* p) {
  Group<V> g;
  if constexpr (V == 4) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
    g.v[0] = q.x; g.v[1] = q.y; g.v[2] = q.z; g.v[3] = q.w;
  } else {
    g.v[0] = __ldg(p);
  }
  return g;
}

// Softmax: y = exp(x - max) / sum exp(x - max).  RMSNorm: y = x * rsqrt(mean x^2 + eps) * gamma.
// Staged: the row lives in dynamic shared memory between passes (width <= kRowStageFloats).
template <bool Softmax, bool Staged, int V>
__global__ void __launch_bounds__(1024) row_stream_kernel(const float* in, const float* gamma, float* out,
                                                          uint64_t rows, int width, uint64_t iterations) {
  extern __shared__ float4 stage4[];
  __shared__ float red[2][kMaxWarps];
  Group<V>* stage = reinterpret_cast<Group<V>*>(stage4);
  const int groups = width / V, T = blockDim.x, t = threadIdx.x;
  int parity = 0;
  for (uint64_t r = 0; r < iterations; ++r) {
    for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
      const float* x = in + row * uint64_t(width);
      float* y = out + row * uint64_t(width);
      // pass 1: load (and stage) this thread's groups; running max or sum of squares
      float acc = Softmax ? -__int_as_float(0x7f800000) : 0.0f;
      int g = t;
      for (; g + 3 * T < groups; g += 4 * T) {
        Group<V> a[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) a[k] = load_group<V>(x + (g + k * T) * V);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if constexpr (Staged) stage[g + k * T] = a[k];
#pragma unroll
          for (int e = 0; e < V; ++e) acc = Softmax ? fmaxf(acc, a[k].v[e]) : acc + a[k].v[e] * a[k].v[e];
        }
      }
      for (; g < groups; g += T) {
        const Group<V> a = load_group<V>(x + g * V);
        if constexpr (Staged) stage[g] = a;
#pragma unroll
        for (int e = 0; e < V; ++e) acc = Softmax ? fmaxf(acc, a.v[e]) : acc + a.v[e] * a.v[e];
      }
      if constexpr (Softmax) {
        const float maximum = cta_reduce<true>(acc, red[parity]);
        parity ^= 1;
        // pass 2: e = exp(x - max), kept in the staged row; sum
        float sum = 0.0f;
        for (g = t; g < groups; g += T) {
          Group<V> a = Staged ? stage[g] : load_group<V>(x + g * V);
#pragma unroll
          for (int e = 0; e < V; ++e) { a.v[e] = expf(a.v[e] - maximum); sum += a.v[e]; }
          if constexpr (Staged) stage[g] = a;
        }
        const float total = cta_reduce<false>(sum, red[parity]);
        parity ^= 1;
        const float scale = 1.0f / total;
        // pass 3: y = e * scale
        for (g = t; g < groups; g += T) {
          Group<V> a;
          if constexpr (Staged) {
            a = stage[g];
          } else {
            a = load_group<V>(x + g * V);
#pragma unroll
            for (int e = 0; e < V; ++e) a.v[e] = expf(a.v[e] - maximum);
          }
#pragma unroll
          for (int e = 0; e < V; ++e) a.v[e] *= scale;
          store_group<V>(y + g * V, a);
        }
      } else {
        const float total = cta_reduce<false>(acc, red[parity]);
        parity ^= 1;
        const float scale = rsqrtf(total / float(width) + kRmsEpsilon);
        // pass 2: y = x * scale * gamma
        for (g = t; g < groups; g += T) {
          Group<V> a = Staged ? stage[g] : load_group<V>(x + g * V);
          const Group<V> w = gamma_group<V>(gamma + g * V);
#pragma unroll
          for (int e = 0; e < V; ++e) a.v[e] = a.v[e] * scale * w.v[e];
          store_group<V>(y + g * V, a);
        }
      }
    }
  }
}

// One warp per row, K quads per lane (width <= 128 K, width % 4 == 0).  With 8
// quads the row needs more than the 64 registers a 1024-thread block leaves a
// thread, so that variant is built for blocks of at most 512 threads.
constexpr int kWarpRowMaxThreads8 = 512;

template <bool Softmax, int K, int MaxThreads = (K == 8 ? kWarpRowMaxThreads8 : 1024)>
__global__ void __launch_bounds__(MaxThreads, 1) row_warp_kernel(const float* in, const float* gamma, float* out,
                                                        uint64_t rows, int width, uint64_t iterations) {
  const int lane = threadIdx.x & 31, quads = width >> 2;
  const uint64_t first = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint64_t warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
  for (uint64_t r = 0; r < iterations; ++r) {
    for (uint64_t row = first; row < rows; row += warps) {
      const float* x = in + row * uint64_t(width);
      float* y = out + row * uint64_t(width);
      float v[K][4];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int q = lane + 32 * k;
        if (q < quads) {
          const uint4 u = ld_cg4(x + 4 * q);
          v[k][0] = __uint_as_float(u.x); v[k][1] = __uint_as_float(u.y);
          v[k][2] = __uint_as_float(u.z); v[k][3] = __uint_as_float(u.w);
        }
      }
      float scale;
      if constexpr (Softmax) {
        float m = -__int_as_float(0x7f800000);
#pragma unroll
        for (int k = 0; k < K; ++k)
          if (lane + 32 * k < quads) m = fmaxf(fmaxf(m, fmaxf(v[k][0], v[k][1])), fmaxf(v[k][2], v[k][3]));
        m = warp_max(m);
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < K; ++k)
          if (lane + 32 * k < quads) {
#pragma unroll
            for (int e = 0; e < 4; ++e) { v[k][e] = expf(v[k][e] - m); sum += v[k][e]; }
          }
        scale = 1.0f / warp_sum(sum);
      } else {
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < K; ++k)
          if (lane + 32 * k < quads) {
#pragma unroll
            for (int e = 0; e < 4; ++e) ss += v[k][e] * v[k][e];
          }
        scale = rsqrtf(warp_sum(ss) / float(width) + kRmsEpsilon);
      }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int q = lane + 32 * k;
        if (q < quads) {
          float o[4];
          if constexpr (Softmax) {
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] = v[k][e] * scale;
          } else {
            const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + q);
            o[0] = v[k][0] * scale * g.x; o[1] = v[k][1] * scale * g.y;
            o[2] = v[k][2] * scale * g.z; o[3] = v[k][3] * scale * g.w;
          }
          st_cg4(y + 4 * q, make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]),
                                       __float_as_uint(o[3])));
        }
      }
    }
  }
}

// One CTA per row with the row in registers: R quads per thread (width a
// multiple of 4, at most 4 R threads floats).  The cross-warp step reads the
// warps' partials as float4s from buffers padded with the reduction's
// identity, so every thread combines them in the same fixed order.
template <bool Max>
__device__ __forceinline__ float cta_reduce_padded(float v, float* red) {
  v = Max ? warp_max(v) : warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const int groups = ((blockDim.x >> 5) + 3) >> 2;
  const float4* r4 = reinterpret_cast<const float4*>(red);
  float r = Max ? -__int_as_float(0x7f800000) : 0.0f;
  for (int g = 0; g < groups; ++g) {
    const float4 q = r4[g];
    r = Max ? fmaxf(fmaxf(fmaxf(r, q.x), q.y), fmaxf(q.z, q.w)) : ((r + q.x) + q.y) + (q.z + q.w);
  }
  return r;
}

template <bool Softmax, int R>
__global__ void __launch_bounds__(1024) row_cta_kernel(const float* in, const float* gamma, float* out,
                                                       uint64_t rows, int width, uint64_t iterations) {
  __shared__ __align__(16) float red[2][kMaxWarps];
  const int quads = width >> 2, t = threadIdx.x, T = blockDim.x;
  for (int i = t; i < 2 * kMaxWarps; i += T) red[i / kMaxWarps][i % kMaxWarps] = (Softmax && i < kMaxWarps) ? -__int_as_float(0x7f800000) : 0.0f;
  __syncthreads();
  int parity = 0;
  for (uint64_t r = 0; r < iterations; ++r) {
    for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
      const float* x = in + row * uint64_t(width);
      float* y = out + row * uint64_t(width);
      float v[R][4];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        const int q = t + k * T;
        if (q < quads) {
          const uint4 u = ld_cg4(x + 4 * q);
          v[k][0] = __uint_as_float(u.x); v[k][1] = __uint_as_float(u.y);
          v[k][2] = __uint_as_float(u.z); v[k][3] = __uint_as_float(u.w);
        }
      }
      float scale;
      if constexpr (Softmax) {
        float m = -__int_as_float(0x7f800000);
#pragma unroll
        for (int k = 0; k < R; ++k)
          if (t + k * T < quads) m = fmaxf(fmaxf(m, fmaxf(v[k][0], v[k][1])), fmaxf(v[k][2], v[k][3]));
        m = cta_reduce_padded<true>(m, red[0]);
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < R; ++k)
          if (t + k * T < quads) {
#pragma unroll
            for (int e = 0; e < 4; ++e) { v[k][e] = expf(v[k][e] - m); sum += v[k][e]; }
          }
        scale = 1.0f / cta_reduce_padded<false>(sum, red[1]);
      } else {
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < R; ++k)
          if (t + k * T < quads) {
#pragma unroll
            for (int e = 0; e < 4; ++e) ss += v[k][e] * v[k][e];
          }
        scale = rsqrtf(cta_reduce_padded<false>(ss, red[parity]) / float(width) + kRmsEpsilon);
        parity ^= 1;
      }
#pragma unroll
      for (int k = 0; k < R; ++k) {
        const int q = t + k * T;
        if (q < quads) {
          float o[4];
          if constexpr (Softmax) {
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] = v[k][e] * scale;
          } else {
            const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + q);
            o[0] = v[k][0] * scale * g.x; o[1] = v[k][1] * scale * g.y;
            o[2] = v[k][2] * scale * g.z; o[3] = v[k][3] * scale * g.w;
          }
          st_cg4(y + 4 * q, make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]),
                                       __float_as_uint(o[3])));
        }
      }
    }
  }
}

// ---------------------------------------------------------------- paired control
// The integer issue loop of the paired reference without per-CTA admission
// counters (gpu_bench.cu:420-430 arithmetic).
__global__ void control_plain_kernel(uint32_t* sink, uint64_t iterations) {
  const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t a = random_word(tid), b = a + 1U, c = a + 2U, d = a + 3U;
  for (uint64_t i = 0; i < iterations; ++i) {
    asm volatile("add.u32 %0, %0, %4;\n\txor.b32 %1, %1, %0;\n\tadd.u32 %2, %2, %1;\n\txor.b32 %3, %3, %2;"
                 : "+r"(a), "+r"(b), "+r"(c), "+r"(d) : "r"(uint32_t(i)));
  }
  sink[tid] = a ^ b ^ c ^ d;
}

// ---------------------------------------------------------------- dispatch
bool staged_row(int width) { return width <= kRowStageFloats; }

template <bool Softmax, bool Staged, int V>
const void* row_handle() { return reinterpret_cast<const void*>(row_stream_kernel<Softmax, Staged, V>); }

// Row-kernel variant: bit 2 softmax, bit 1 staged, bit 0 16-byte groups.
int row_variant(int fn, int width) {
  return (fn == NL_SOFTMAX ? 4 : 0) | (staged_row(width) ? 2 : 0) | (width % 4 == 0 ? 1 : 0);
}

// Quads per lane of the warp-per-row layout, or 0 when a CTA must own each row:
// rows wider than 1024 floats or not a multiple of 4, or fewer rows than warps.
int warp_row_quads(int width, uint64_t rows, int blocks, int threads) {
  if (width % 4 || width > 1024 || uint64_t(blocks) * uint64_t(threads / 32) > rows) return 0;
  if (width > 512 && threads > kWarpRowMaxThreads8) return 0;
  return width <= 128 ? 1 : width <= 256 ? 2 : width <= 512 ? 4 : 8;
}

// Quads per thread of the register CTA-per-row layout, or 0: rows not a
// multiple of 4 or wider than 16 x threads floats.
int cta_row_quads(int width, int threads) {
  if (width % 4) return 0;
  const int per_thread = (width / 4 + threads - 1) / threads;
  return per_thread <= 1 ? 1 : per_thread <= 2 ? 2 : per_thread <= 4 ? 4 : 0;
}

template <bool Softmax>
const void* cta_row_handle(int r) {
  switch (r) {
    case 1: return reinterpret_cast<const void*>(row_cta_kernel<Softmax, 1>);
    case 2: return reinterpret_cast<const void*>(row_cta_kernel<Softmax, 2>);
    default: return reinterpret_cast<const void*>(row_cta_kernel<Softmax, 4>);
  }
}

template <bool Softmax>
const void* warp_row_handle(int k) {
  switch (k) {
    case 1: return reinterpret_cast<const void*>(row_warp_kernel<Softmax, 1>);
    case 2: return reinterpret_cast<const void*>(row_warp_kernel<Softmax, 2>);
    case 4: return reinterpret_cast<const void*>(row_warp_kernel<Softmax, 4>);
    default: return reinterpret_cast<const void*>(row_warp_kernel<Softmax, 8>);
  }
}

const void* row_kernel(int fn, int width) {
  switch (row_variant(fn, width)) {
    case 7: return row_handle<true, true, 4>();
    case 6: return row_handle<true, true, 1>();
    case 5: return row_handle<true, false, 4>();
    case 4: return row_handle<true, false, 1>();
    case 3: return row_handle<false, true, 4>();
    case 2: return row_handle<false, true, 1>();
    case 1: return row_handle<false, false, 4>();
    default: return row_handle<false, false, 1>();
  }
}

std::atomic<int> g_row_smem_limit[8][kMaxDevices];

}  // namespace

NonlinearLayout nonlinear_layout(int fn, uint64_t n, int width, int blocks, int threads) {
  NonlinearLayout l{};
  switch (fn) {
    case NL_EXP: l.kernel = reinterpret_cast<const void*>(pointwise_stream_kernel<NL_EXP>); break;
    case NL_TANH: l.kernel = reinterpret_cast<const void*>(pointwise_stream_kernel<NL_TANH>); break;
    case NL_SILU: l.kernel = reinterpret_cast<const void*>(pointwise_stream_kernel<NL_SILU>); break;
    default: {
      const int k = warp_row_quads(width, n / uint64_t(width), blocks, threads);
      const int r = cta_row_quads(width, threads);
      if (k) {
        l.kernel = fn == NL_SOFTMAX ? warp_row_handle<true>(k) : warp_row_handle<false>(k);
        l.warp_rows = true;
      } else if (r) {
        l.kernel = fn == NL_SOFTMAX ? cta_row_handle<true>(r) : cta_row_handle<false>(r);
        l.cta_registers = true;
      } else {
        l.kernel = row_kernel(fn, width);
        l.dynamic_smem = staged_row(width) ? size_t(width) * 4 : 0;
      }
    }
  }
  l.description = fn < NL_SOFTMAX ? "grid-stride 16-byte quads, four in flight per thread; scalar tail"
                  : l.warp_rows ? "one warp per row, row in registers (16-byte groups); warp-shuffle reductions"
                  : l.cta_registers ? "one CTA per row, row in registers (16-byte groups); warp-shuffle reductions"
                  : l.dynamic_smem ? "one CTA per row, row staged once in shared memory; warp-shuffle reductions"
                  : "one CTA per row, row re-read from global memory per pass; warp-shuffle reductions";
  return l;
}

cudaError_t launch_nonlinear_fill(float* data, uint64_t n, uint64_t seed, float shift, int gamma, int sms, cudaStream_t s) {
  if (!n) return cudaSuccess;
  const uint64_t want = (n + 255) / 256;
  const int blocks = int(want < uint64_t(sms) * 8 ? want : uint64_t(sms) * 8);
  nonlinear_fill_kernel<<<blocks, 256, 0, s>>>(data, n, seed, shift, gamma);
  return cudaGetLastError();
}

cudaError_t launch_nonlinear(int fn, const float* in, const float* gamma, float* out, uint64_t n, int width,
                             uint64_t iterations, int blocks, int threads, cudaStream_t s) {
  if (fn == NL_EXP) pointwise_stream_kernel<NL_EXP><<<blocks, threads, 0, s>>>(in, out, n, iterations);
  else if (fn == NL_TANH) pointwise_stream_kernel<NL_TANH><<<blocks, threads, 0, s>>>(in, out, n, iterations);
  else if (fn == NL_SILU) pointwise_stream_kernel<NL_SILU><<<blocks, threads, 0, s>>>(in, out, n, iterations);
  else {
    const NonlinearLayout l = nonlinear_layout(fn, n, width, blocks, threads);
    if (!l.warp_rows && !l.cta_registers)
      ensure_dynamic_smem(l.kernel, 2 * kMaxWarps * sizeof(float), l.dynamic_smem, g_row_smem_limit[row_variant(fn, width)]);
    const uint64_t rows = n / uint64_t(width);
    void* args[] = {&in, &gamma, &out, const_cast<uint64_t*>(&rows), &width, &iterations};
    return cudaLaunchKernel(l.kernel, dim3(blocks), dim3(threads), args, l.dynamic_smem, s);
  }
  return cudaGetLastError();
}

cudaError_t launch_control_plain(uint32_t* sink, uint64_t iterations, int blocks, int threads, cudaStream_t s) {
  control_plain_kernel<<<blocks, threads, 0, s>>>(sink, iterations);
  return cudaGetLastError();
}

const void* control_plain_handle() { return reinterpret_cast<const void*>(control_plain_kernel); }

}  // namespace pm

using namespace pm;

extern "C" int pm_nonlinear_fill_device(float* data, uint64_t n, uint64_t seed, float shift, int gamma, void* stream) {
  if (!data && n) return fail(PM_E_INVALID, "pm_nonlinear_fill_device: NULL buffer");
  int device = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return cuda_fail(e, "pm_nonlinear_fill_device");
  e = launch_nonlinear_fill(data, n, seed, shift, gamma ? 1 : 0, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PM_OK : cuda_fail(e, "pm_nonlinear_fill_device launch");
}

extern "C" int pm_nonlinear_apply_device(int32_t function, const float* input, const float* gamma, float* output, uint64_t n,
                                         int32_t row_width, uint64_t iterations, int32_t blocks, int32_t threads,
                                         void* stream) {
  if (function < PM_NL_EXP || function > PM_NL_RMSNORM) return fail(PM_E_INVALID, "pm_nonlinear_apply_device: unknown function");
  const bool rowwise = function == PM_NL_SOFTMAX || function == PM_NL_RMSNORM;
  if (!input || !output || !n) return fail(PM_E_INVALID, "pm_nonlinear_apply_device: empty input or NULL buffer");
  if ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output) |
       reinterpret_cast<uintptr_t>(function == PM_NL_RMSNORM ? gamma : nullptr)) & 15)
    return fail(PM_E_INVALID, "pm_nonlinear_apply_device: buffers must be 16-byte aligned");
  if (threads < 32 || threads > 1024 || threads % 32) return fail(PM_E_INVALID, "pm_nonlinear_apply_device: threads must be a multiple of 32 in 32..1024");
  if (blocks < 1 || blocks > 1000000) return fail(PM_E_INVALID, "pm_nonlinear_apply_device: blocks must be in 1..1000000");
  if (iterations > (1ULL << 32)) return fail(PM_E_LIMIT, "pm_nonlinear_apply_device: iterations must be <= 2^32");
  if (rowwise && (row_width < 1 || row_width > 65536 || n % uint64_t(row_width)))
    return fail(PM_E_INVALID, "pm_nonlinear_apply_device: softmax/RMSNorm need complete rows of width 1..65536");
  if (!rowwise && row_width) return fail(PM_E_INVALID, "pm_nonlinear_apply_device: row_width applies only to softmax/RMSNorm");
  if (function == PM_NL_RMSNORM && !gamma) return fail(PM_E_INVALID, "pm_nonlinear_apply_device: RMSNorm needs gamma");
  const cudaError_t e = launch_nonlinear(function, input, gamma, output, n, row_width, iterations, blocks, threads,
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PM_OK : cuda_fail(e, "pm_nonlinear_apply_device launch");
}
