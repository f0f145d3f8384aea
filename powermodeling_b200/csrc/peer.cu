// Peer buffers (CUDA IPC) and the bounded arrival wait of the row exchange
// (include/pmb200_peer.h).  The row stores themselves are the analysis
// kernel's epilogue (analysis.cu, deliver_rows).
#include <cuda_runtime.h>
#include <cstring>

#include "pmb200.h"
#include "pmb200_peer.h"
#include "pm_capi.h"

namespace pm {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread r polls rank r's flag at system scope until it reaches `epoch`
// (wrap-safe compare) or `timeout_ns` passes; then it records the error and
// stops waiting.
__global__ void peer_wait_kernel(const uint32_t* flags, int n, uint32_t epoch, uint64_t timeout_ns, int32_t* error) {
  const int r = threadIdx.x;
  if (r < n) {
    const uint64_t t0 = global_ns();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (global_ns() - t0 > timeout_ns) { atomicExch(error, 1); break; }
      __nanosleep(256);
    }
  }
  __syncthreads();
}

// The start line: thread 0 stores `epoch` into this rank's entry of every
// rank's flag array, then thread r polls entry r of this rank's own array,
// as peer_wait_kernel does.
struct GateFlags {
  uint32_t* flags[PM_MAX_RANKS];
};

__global__ void peer_gate_kernel(GateFlags F, int n, int rank, uint32_t epoch, uint64_t timeout_ns, int32_t* error) {
  if (threadIdx.x == 0)
    for (int r = 0; r < n; ++r)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(F.flags[r] + rank), "r"(epoch) : "memory");
  const int r = threadIdx.x;
  if (r < n) {
    const uint32_t* own = F.flags[rank];
    const uint64_t t0 = global_ns();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(own + r) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (global_ns() - t0 > timeout_ns) { atomicExch(error, 1); break; }
      __nanosleep(256);
    }
  }
  __syncthreads();
}

}  // namespace pm

using namespace pm;

extern "C" {

int pm_peer_alloc(size_t bytes, void** device_ptr, pm_peer_handle* handle) {
  if (!device_ptr || !handle || bytes == 0) return fail(PM_E_INVALID, "pm_peer_alloc: bad argument");
  int device = 0, rc = current_device(&device);
  if (rc) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(peer buffer)");
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer buffer export");
  }
  static_assert(sizeof(h) <= sizeof(handle->bytes), "IPC handle size");
  memset(handle->bytes, 0, sizeof(handle->bytes));
  memcpy(handle->bytes, &h, sizeof(h));
  *device_ptr = p;
  return PM_OK;
}

int pm_peer_free(void* device_ptr) {
  if (!device_ptr) return PM_OK;
  const cudaError_t e = cudaFree(device_ptr);
  return e == cudaSuccess ? PM_OK : cuda_fail(e, "cudaFree(peer buffer)");
}

int pm_peer_open(const pm_peer_handle* handle, void** device_ptr) {
  if (!handle || !device_ptr) return fail(PM_E_INVALID, "pm_peer_open: NULL argument");
  int device = 0, rc = current_device(&device);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? PM_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int pm_peer_close(void* device_ptr) {
  if (!device_ptr) return PM_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(device_ptr);
  return e == cudaSuccess ? PM_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int pm_peer_wait_device(const uint32_t* flags, int32_t n_ranks, uint32_t epoch, uint32_t timeout_ms, int32_t* error,
                        void* stream) {
  if (!flags || !error || n_ranks < 1 || n_ranks > PM_MAX_RANKS) return fail(PM_E_INVALID, "pm_peer_wait_device: bad argument");
  peer_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flags, n_ranks, epoch, (uint64_t)timeout_ms * 1000000ull, error);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e, "peer_wait_kernel launch");
}

int pm_peer_gate_device(uint32_t* const* flags, int32_t n_ranks, int32_t rank, uint32_t epoch, uint32_t timeout_ms,
                        int32_t* error, void* stream) {
  if (!flags || !error || n_ranks < 1 || n_ranks > PM_MAX_RANKS || rank < 0 || rank >= n_ranks)
    return fail(PM_E_INVALID, "pm_peer_gate_device: bad argument");
  GateFlags F{};
  for (int r = 0; r < n_ranks; ++r) {
    if (!flags[r]) return fail(PM_E_INVALID, "pm_peer_gate_device: rank %d's flags are NULL", r);
    F.flags[r] = flags[r];
  }
  peer_gate_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(F, n_ranks, rank, epoch, (uint64_t)timeout_ms * 1000000ull, error);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PM_OK : cuda_fail(e, "peer_gate_kernel launch");
}

}  // extern "C"
