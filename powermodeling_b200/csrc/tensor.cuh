// Dense FP16 -> FP32 tensor arms on sm_100a (tcgen05 / TMEM, operands via TMA).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "workloads.cuh"

namespace pm {

// Tile of the register-reuse analog: one CTA holds A (128 x 64) and B (N x 64),
// both K-major fp16 in 128-byte-swizzled shared memory, loaded once by TMA,
// and issues tcgen05.mma.kind::f16 (M=128, K=16 per instruction) into
// `accumulators` independent TMEM tiles of N columns each.
constexpr int kTmaM = 128, kTmaK = 64;
int tensor_tile_n(int accumulators);                    // N per accumulator (<= 256, 512 TMEM columns total)
double tensor_flops_per_iteration(int accumulators);    // per CTA: accumulators * 4 MMAs * 2*M*N*16

struct TensorStatus {                                   // written by the kernel
  unsigned int timeouts;                                // bounded waits that gave up
  unsigned int done_ctas;
};

// a: 128 x 64 fp16 (K-major), b: 256 x 64 fp16 (K-major); out receives the
// first accumulator of every admitted CTA (128 x N fp32).
cudaError_t launch_tensor_mma(const void* a, const void* b, float* out, uint64_t iterations, int accumulators,
                              int blocks, int threads, Admission adm, TensorStatus* status, cudaStream_t s);
cudaError_t tensor_mma_attributes(int accumulators, cudaFuncAttributes* attr);

}  // namespace pm
