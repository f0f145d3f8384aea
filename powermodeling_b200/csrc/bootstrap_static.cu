// Group bootstrap for callers that must not allocate device memory.
//
// Some callers cannot let a library call cudaMalloc: a host process that has
// already handed every byte of the device to its own memory pool, an
// allocator-owning runtime that forbids foreign allocations on its device,
// or a service that must bound the library's footprint in advance.  For
// them pm_group_bootstrap_device_static runs the same bootstrap kernel as
// pm_group_bootstrap_device, but the index streams of groups with more than
// seven members live in a fixed array compiled into this library
// (kStaticStreamBytes, held by every GPU that loads the library until the
// process exits) instead of a caller-provided scratch buffer.  Inputs and
// outputs are still the caller's device buffers.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "pmb200.h"
#include "pmb200_peer.h"
#include "pm_capi.h"

namespace pm {

int launch_bootstrap(const BootArgs& A, cudaStream_t stream, const pm_peer_groups* groups = nullptr);
int launch_bootstrap_prepare(const BootArgs& A, cudaStream_t stream);
int prepare_bootstrap_constants(int device);

namespace {

// Prepared multiset histograms (6.9 KB per group) and index streams
// (resamples x max_members bytes per group; for groups of up to seven members
// only while they fit, the faster prepare pass): 32 MiB covers, for example,
// 4800 groups of up to seven members, or 200 groups of up to 16 members at
// 10 000 resamples.
constexpr size_t kStaticStreamBytes = size_t(32) << 20;
static __device__ __align__(256) uint8_t g_static_streams[kStaticStreamBytes];

// Device address of g_static_streams per device.  In host code the symbol
// name is only a stand-in; the address must come from cudaGetSymbolAddress
// with that device current.
void* g_static_address[kMaxDevices] = {};
std::mutex g_static_lock;

}  // namespace
}  // namespace pm

using namespace pm;

extern "C" size_t pm_bootstrap_static_scratch_capacity(void) { return kStaticStreamBytes; }

extern "C" int pm_group_bootstrap_device_static(const pm_bootstrap_job* job, void* stream) {
  // The checks of every other bootstrap entry point (sizes, limits, arrays).
  int rc = check_bootstrap(job);
  if (rc) return rc;
  // Every group's index stream when the array holds them (the faster prepare
  // pass), else only what the fused pass needs.
  const bool streamed = bootstrap_scratch_bytes(job->n_groups, job->max_members, job->resamples) <= kStaticStreamBytes;
  const size_t need = bootstrap_scratch_bytes(job->n_groups, job->max_members, job->resamples, streamed);
  if (need > kStaticStreamBytes)
    return fail(PM_E_LIMIT,
                "pm_group_bootstrap_device_static: %d groups of up to %d members at %d resamples need %zu bytes of "
                "index streams; the fixed array holds %zu (use pm_group_bootstrap_device with your own scratch)",
                job->n_groups, job->max_members, job->resamples, need, kStaticStreamBytes);
  int device = 0;
  if ((rc = current_device(&device))) return rc;
  if ((rc = check_bootstrap_fits(job->n_metrics, job->max_members))) return rc;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> guard(g_static_lock);
    if (!g_static_address[device]) {
      // Once per device, with that device current: the array's device address.
      cudaError_t e = cudaGetSymbolAddress(&g_static_address[device], g_static_streams);
      if (e != cudaSuccess) {
        g_static_address[device] = nullptr;
        return cuda_fail(e, "cudaGetSymbolAddress(g_static_streams)");
      }
    }
    scratch = g_static_address[device];
  }
  if (prepare_bootstrap_constants(device)) return fail(PM_E_CUDA, "bootstrap constants upload failed");
  // Nothing in the array must start at zero: the prepare launch writes each
  // group's histogram or stream completely before the fold reads it back.
  BootArgs A{job->n_groups, job->n_metrics, job->resamples, job->max_members, job->values, job->group_offsets,
             job->member_rows, job->member_valid, job->seeds, job->medians, job->ci_lo, job->ci_hi,
             static_cast<uint8_t*>(scratch), 1, streamed ? 1 : 0};
  if (launch_bootstrap_prepare(A, static_cast<cudaStream_t>(stream)))
    return fail(PM_E_CUDA, "bootstrap_prepare_kernel launch failed");
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_prepare_kernel launch");
  if (launch_bootstrap(A, static_cast<cudaStream_t>(stream))) return fail(PM_E_CUDA, "bootstrap_kernel launch failed");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_kernel launch");
  return PM_OK;
}
