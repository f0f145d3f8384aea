// Dense FP16 -> FP32 operand-reuse tensor arm on sm_100a: tcgen05.mma with
// TMEM accumulators, operands staged once by TMA.
//
// The reference's tensor arm (cuda/gpu_bench.cu:434-455) keeps one WMMA
// 16x16x16 A/B fragment pair in registers per warp and loops mma_sync on 1-8
// independent accumulators.  Here a CTA stages A (128 x 64) and B (N x 64),
// K-major fp16 with the 128-byte swizzle, into shared memory with one TMA
// load each; a single elected thread then issues
// tcgen05.mma.cta_group::1.kind::f16 (M=128, K=16) `iterations` x
// `accumulators` x 4 times, rotating over `accumulators` TMEM tiles of N fp32
// columns, commits to an mbarrier, and the four warps read accumulator 0 back
// with tcgen05.ld.  Every wait is bounded by %globaltimer; on expiry the
// kernel records a timeout, waits (bounded) for its MMAs, frees TMEM and
// returns.  Every load is a plain per-CTA TMA copy.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "tensor.cuh"

namespace pm {

int tensor_tile_n(int accumulators) {
  int n = (512 / accumulators) / 16 * 16;
  return n > 256 ? 256 : n;
}
double tensor_flops_per_iteration(int accumulators) {
  return double(accumulators) * 4.0 * 2.0 * kTmaM * tensor_tile_n(accumulators) * 16.0;
}

namespace {

constexpr int kATileBytes = kTmaM * kTmaK * 2;            // 16 KiB
constexpr uint64_t kWaitNs = 20ull * 1000000000ull;        // bound on any single wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(done) : "r"(bar), "r"(parity) : "memory");
  return done != 0;
}
// Spin on an mbarrier phase until it completes or `deadline` (globaltimer ns) passes.
__device__ __forceinline__ bool mbar_wait_until(uint32_t bar, uint32_t parity, uint64_t deadline) {
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() > deadline) return false;
  return true;
}

// K-major, 128-byte swizzled operand: rows of 128 B, 8-row atoms of 1 KiB.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3fff);            // start address
  d |= uint64_t(1) << 16;                         // leading byte offset (unused with swizzle)
  d |= uint64_t(1024 >> 4) << 32;                 // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                         // descriptor version for tcgen05
  d |= uint64_t(2) << 61;                         // layout: 128-byte swizzle
  return d;
}

__device__ __forceinline__ uint32_t instr_desc_f16(int n) {
  return (1u << 4)                                // D format: f32
         | (uint32_t(n >> 3) << 17)               // N
         | (uint32_t(kTmaM >> 4) << 24);          // M = 128; A, B f16 and K-major (zero fields)
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
               :: "r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ unsigned smid_t() {
  unsigned id;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(id));
  return id;
}

__global__ void __launch_bounds__(256)
tensor_mma_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, float* out,
                  uint64_t iterations, int accumulators, int n, Admission adm, TensorStatus* status) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;
  __shared__ int admitted;
  if (threadIdx.x == 0) {
    const unsigned id = smid_t();
    admitted = id < kSmSlots && (!adm.filtered || adm.mask[id]);
    if (admitted) atomicAdd(adm.blocks_per_sm + id, 1ULL);
  }
  __syncthreads();
  if (!admitted) return;
  // 1024-byte aligned operand tiles (the 128-byte swizzle is computed from address bits).
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* tile_a = base;
  unsigned char* tile_b = base + kATileBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int cols = 32;
  while (cols < accumulators * n) cols <<= 1;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(&tmem_base)), "r"(cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  const uint32_t bl = smem_u32(&bar_load), bm = smem_u32(&bar_mma);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(bl) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(bm) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  bool ok = true;
  if (threadIdx.x == 0) {
    const uint32_t bytes = uint32_t(kATileBytes + n * kTmaK * 2);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bl), "r"(bytes) : "memory");
    const int x = 0, y = 0;
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(smem_u32(tile_a)), "l"(&map_a), "r"(x), "r"(y), "r"(bl) : "memory");
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(smem_u32(tile_b)), "l"(&map_b), "r"(x), "r"(y), "r"(bl) : "memory");
    ok = mbar_wait_until(bl, 0, globaltimer() + kWaitNs);
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t da = smem_desc(smem_u32(tile_a)), db = smem_desc(smem_u32(tile_b));
      const uint32_t idesc = instr_desc_f16(n);
      for (uint64_t it = 0; it < iterations; ++it)
        for (int j = 0; j < accumulators; ++j)
#pragma unroll
          for (int k = 0; k < kTmaK / 16; ++k)   // K slices of 16 fp16 = 32 bytes = 2 descriptor units
            mma_f16(tmem + uint32_t(j * n), da + uint64_t(2 * k), db + uint64_t(2 * k), idesc, (it | k) ? 1u : 0u);
    } else {
      atomicAdd(&status->timeouts, 1u);
    }
    // Commit even on a failed load so bar_mma completes once pending MMAs (if any) drain.
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bm) : "memory");
  }
  const bool mma_done = mbar_wait_until(bm, 0, globaltimer() + kWaitNs);
  if (!mma_done && lane == 0) atomicAdd(&status->timeouts, 1u);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (mma_done && warp < 4) {
    // Accumulator 0 -> out[block][row][col]; warp w owns TMEM lanes 32w..32w+31.
    float* row = out + (size_t(blockIdx.x) * kTmaM + size_t(warp * 32 + lane)) * n;
    for (int c = 0; c < n; c += 8) {
      uint32_t v[8];
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                   : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                   : "r"(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c)));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      float4* dst = reinterpret_cast<float4*>(row + c);
      dst[0] = make_float4(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]), __uint_as_float(v[3]));
      dst[1] = make_float4(__uint_as_float(v[4]), __uint_as_float(v[5]), __uint_as_float(v[6]), __uint_as_float(v[7]));
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(cols) : "memory");
  }
  if (threadIdx.x == 0 && mma_done) atomicAdd(&status->done_ctas, 1u);
}

// ---------------------------------------------------------------- host
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                 const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// K-major fp16 matrix of `rows` x 64, box of `box_rows` x 64 with the 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cuuint64_t(kTmaK), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(kTmaK) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kTmaK), box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t tensor_smem_bytes(int n) { return size_t(kATileBytes) + size_t(n) * kTmaK * 2 + 1024; }

cudaError_t launch_tensor_mma(const void* a, const void* b, float* out, uint64_t iterations, int accumulators, int blocks,
                              int threads, Admission adm, TensorStatus* status, cudaStream_t s) {
  if (accumulators < 1 || accumulators > 8 || (threads != 128 && threads != 256)) return cudaErrorInvalidValue;
  const int n = tensor_tile_n(accumulators);
  CUtensorMap ma, mb;
  if (!make_map(&ma, a, kTmaM, kTmaM) || !make_map(&mb, b, 256, uint32_t(n))) return cudaErrorInvalidValue;
  const size_t smem = tensor_smem_bytes(n);
  cudaError_t e = cudaFuncSetAttribute(tensor_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  tensor_mma_kernel<<<blocks, threads, smem, s>>>(ma, mb, out, iterations, accumulators, n, adm, status);
  return cudaGetLastError();
}

cudaError_t tensor_mma_attributes(int accumulators, cudaFuncAttributes* attr) {
  (void)accumulators;
  return cudaFuncGetAttributes(attr, tensor_mma_kernel);
}

}  // namespace pm
