// Workload kernels of the measured arms (declarations and shared device helpers).
//
// The deterministic word fill, the per-thread read-sum semantics, the
// four-stream write/copy streams, the integer issue loop, the dependent
// chase and the SFU recurrence reproduce the reference's observable results
// (cuda/gpu_bench.cu:277-473, cuda/sfu.cuh:43-117) so checksums and terminal
// indices compare bit for bit; the vector (16-byte) read/copy and the
// line-granular chase are additional B200 modes with their own version tags.
#pragma once
#include <cstring>
#include <cstdint>
#include <cuda_runtime.h>

namespace pm {

constexpr unsigned kSmSlots = 4096;          // per-SM admission/telemetry counters

// splitmix64 finaliser (Steele, Lea & Flood 2014) truncated to 32 bits: the
// deterministic payload of every memory buffer (gpu_bench.cu:277-282).
__host__ __device__ __forceinline__ uint32_t random_word(uint64_t x) {
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return uint32_t(x ^ (x >> 31));
}

// First operand of an SFU chain: a [0.5, 1) mantissa from the lane hash (sfu.cuh:73-75).
__host__ __device__ __forceinline__ uint32_t sfu_initial_bits(uint64_t lane, uint64_t seed, int chain) {
  return (random_word(lane ^ seed ^ (uint64_t(chain + 1) * 0x9e3779b97f4a7c15ULL)) & 0x007fffffU) | 0x3f000000U;
}

// Seeded uint32 LCG fill (an extra mode beside random_word): x_0 = low 32 bits
// of the seed, x_{i+1} = 1664525 x_i + 1013904223 (mod 2^32), word i = x_i.
// Word i is reached in at most 64 squarings of the affine step (a, c):
// composing (a1, c1) after (a2, c2) gives (a1 a2, a1 c2 + c1).
__host__ __device__ __forceinline__ uint32_t lcg_word(uint64_t i, uint64_t seed) {
  uint32_t a = 1664525U, c = 1013904223U, x = uint32_t(seed);
  while (i) {
    if (i & 1) x = a * x + c;
    c = a * c + c;
    a = a * a;
    i >>= 1;
  }
  return x;
}
enum WordFill { FILL_RANDOM_WORD = 0, FILL_LCG = 1 };

// The SFU arm's uniform input mode (an extra mode beside the reference's
// [0.5, 1) operand): uniform in [0.5, 2.0) from the thread-index hash,
// 0.5 + 1.5 m / 2^24 for the top 24 bits m of the hash, in two separately
// rounded float operations.
__host__ __device__ __forceinline__ uint32_t sfu_uniform_bits(uint64_t lane, uint64_t seed, int chain) {
  const uint32_t m = random_word(lane ^ seed ^ (uint64_t(chain + 1) * 0x9e3779b97f4a7c15ULL)) >> 8;
  const float scaled = float(m) * (1.5f / 16777216.0f);
  const float x = scaled + 0.5f;
  uint32_t bits;
  memcpy(&bits, &x, 4);
  return bits;
}
enum SfuInput { SFU_INPUT_PARITY = 0, SFU_INPUT_UNIFORM_0P5_2 = 1 };

// Cache policies of the read arms.
enum ReadPolicy { RP_CA = 0, RP_CG = 1, RP_CS = 2 };
enum SfuOp { SFU_EX2 = 0, SFU_TANH = 1, SFU_RSQRT = 2, SFU_RCP = 3, SFU_LG2 = 4, SFU_SQRT = 5 };

struct Admission {
  const unsigned char* mask;      // kSmSlots bytes, 1 = admit blocks dispatched to that SM
  bool filtered;
  unsigned long long* blocks_per_sm;
};

// Host launchers (workloads.cu).  All return cudaGetLastError() of the launch.
cudaError_t launch_fill_words(uint32_t* data, uint64_t n, uint64_t seed, int sms, cudaStream_t s, int fill = FILL_RANDOM_WORD);
cudaError_t launch_fill_halves(void* data, uint64_t n, uint64_t seed, int uniform_pm1, int sms, cudaStream_t s);
cudaError_t launch_read_scalar(int policy, bool l1, const uint32_t* in, uint32_t* sink, uint64_t words, uint64_t slice,
                               uint64_t stride, uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s);
cudaError_t launch_read_vector(int policy, const uint32_t* in, uint32_t* sink, uint64_t quads, uint64_t stride,
                               uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s);
cudaError_t launch_write_copy_scalar(bool copy, const uint32_t* in, uint32_t* out, uint32_t* sink, uint64_t words,
                                     uint64_t stride, uint64_t iterations, int blocks, int threads, Admission adm,
                                     cudaStream_t s);
cudaError_t launch_copy_vector(const uint32_t* in, uint32_t* out, uint32_t* sink, uint64_t quads, uint64_t stride,
                               uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s);
cudaError_t launch_control(uint32_t* sink, uint64_t iterations, int blocks, int threads, Admission adm, cudaStream_t s);
cudaError_t launch_chase_words(const uint32_t* links, uint32_t* sink, uint64_t words, uint64_t iterations, uint64_t nonce,
                               int blocks, int threads, Admission adm, unsigned long long* cycles,
                               unsigned long long* loads, cudaStream_t s);
cudaError_t launch_chase_lines(const uint64_t* lines, uint64_t* terminal, uint64_t nodes, uint64_t iterations,
                               uint64_t nonce, int blocks, int threads, Admission adm, unsigned long long* cycles,
                               unsigned long long* loads, cudaStream_t s);
// input: SFU_INPUT_PARITY (the reference's operands, FNV hash of the chains per lane) or
// SFU_INPUT_UNIFORM_0P5_2 (uniform [0.5, 2.0) operands, XOR of the chains per lane).
cudaError_t launch_sfu(int op, bool control, int chains, uint32_t* sink, uint64_t lanes, uint64_t iterations,
                       uint64_t seed, int blocks, int threads, cudaStream_t s, int input = SFU_INPUT_PARITY);
cudaError_t launch_sfu_check(int op, uint32_t* sample, uint64_t lanes, uint64_t seed, int chains, cudaStream_t s,
                             int input = SFU_INPUT_PARITY);
cudaError_t sfu_attributes(int op, bool control, int chains, cudaFuncAttributes* attr);
const void* kernel_symbol(const char* name, int a, int b, int c);

// Streaming FP32 nonlinear functions (nonlinear.cu; the reference's cuda/nonlinear.cuh).
enum NonlinearFn { NL_EXP = 0, NL_TANH = 1, NL_SILU = 2, NL_SOFTMAX = 3, NL_RMSNORM = 4 };
// Input (gamma = 0: (int(w & 0xffff) - 32768) / 8192 + shift) or RMSNorm gamma
// (gamma = 1: 0.75 + (w & 0xffff) / 131072), w = random_word(i ^ seed).
cudaError_t launch_nonlinear_fill(float* data, uint64_t n, uint64_t seed, float shift, int gamma, int sms, cudaStream_t s);
// `iterations` applications of function fn to n inputs (rows of `width` for
// softmax/RMSNorm) on a blocks x threads grid; in/out 16-byte aligned.
cudaError_t launch_nonlinear(int fn, const float* in, const float* gamma, float* out, uint64_t n, int width,
                             uint64_t iterations, int blocks, int threads, cudaStream_t s);
// The kernel, its dynamic shared memory and a one-line description of how a
// launch of function fn over n inputs on blocks x threads lays out the work.
struct NonlinearLayout { const void* kernel; size_t dynamic_smem; bool warp_rows, cta_registers; const char* description; };
NonlinearLayout nonlinear_layout(int fn, uint64_t n, int width, int blocks, int threads);
// The integer issue loop without admission counters (paired reference of the nonlinear arms).
cudaError_t launch_control_plain(uint32_t* sink, uint64_t iterations, int blocks, int threads, cudaStream_t s);
const void* control_plain_handle();
const void* sfu_kernel_handle(int op, bool control, int chains);

}  // namespace pm
