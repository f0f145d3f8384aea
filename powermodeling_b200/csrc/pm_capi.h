// Host-side declarations shared by the C ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <atomic>
#include <mutex>

#include "pmb200.h"

namespace pm {

constexpr int kMaxDevices = 64;
constexpr int kMaxPhaseSamples = 1 << 24;   // samples in one (trial, phase) segment
constexpr int kMaxEpochsPerArm = 256;
constexpr int kMaxGroupMembers = 128;       // bootstrap rows per group
constexpr int kMaxMetrics = 256;
constexpr int kSortColumns = 18;            // per-phase tile: 10 sample columns + 8 staged columns
constexpr size_t kSmemSortBytes = 160 * 1024;

// Arguments of the group bootstrap kernel.
struct BootArgs {
  int n_groups, n_metrics, resamples, max_members;
  const double* values;
  const int32_t* offsets;
  const int32_t* member_rows;     // NULL: identity
  const uint8_t* member_valid;    // NULL: all rows count
  const uint64_t* seeds;
  double* medians; double* lo; double* hi;
  uint8_t* scratch;               // prepared histograms, then index streams (all groups if streamed, else those above 7 members)
  int prepared;                   // 1: bootstrap_prepare_kernel filled scratch for each group's member count
  int streamed;                   // 1: scratch holds every group's index stream (bootstrap_scratch_bytes(..., true))
};
// Device scratch of a bootstrap: one histogram per group, plus index streams
// for every group (streamed) or only when max_members > 7 (bootstrap.cu).
size_t bootstrap_scratch_bytes(int n_groups, int max_members, int resamples, bool streamed = true);

// Raises `kernel`'s dynamic shared-memory limit on the current device to at
// least `bytes` (static plus dynamic above 48 KB needs the opt-in); `limits`
// remembers each device's current limit so the attribute call is made only
// when it must grow, not on every launch.
template <class Kernel>
void ensure_dynamic_smem(Kernel kernel, size_t static_bytes, size_t bytes, std::atomic<int>* limits) {
  if (static_bytes + bytes <= 48 * 1024) return;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) device = 0;
  if ((int)bytes <= limits[device].load(std::memory_order_relaxed)) return;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess)
    limits[device].store((int)bytes, std::memory_order_relaxed);
}

// Grow-only device workspace, pinned staging buffer and private stream of a device.
struct Arena {
  void* dev = nullptr; size_t dev_bytes = 0;
  void* host = nullptr; size_t host_bytes = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t side = nullptr;                 // work that overlaps the main stream (stream generation)
  cudaEvent_t fork = nullptr, join = nullptr;  // main -> side and side -> main ordering
  cudaEvent_t analysed = nullptr, results = nullptr;   // trial results ready on the device / on the host
  std::mutex lock;
};
extern Arena g_arenas[kMaxDevices];

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* where);
int current_device(int* device);
int arena_reserve(Arena& a, size_t dev_bytes, size_t host_bytes);
size_t bootstrap_smem_shortfall(int n_metrics, int max_members, size_t* available);
// PM_E_LIMIT when the bootstrap fold for these sizes does not fit one CTA's shared memory.
int check_bootstrap_fits(int n_metrics, int max_members);
// PM_E_INVALID / PM_E_LIMIT for a job whose sizes, limits or arrays are unusable.
int check_bootstrap(const pm_bootstrap_job* j);
size_t analyze_scratch_bytes(int n_trials, int max_phase_samples);

}  // namespace pm
