// C ABI of libpmb200 (analysis half): argument checks, staging of host
// buffers through pinned memory, grow-only device workspaces and kernel
// launches.  Nothing here computes a result on the host; every number that
// leaves these functions was produced by a kernel.
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>
#if defined(__x86_64__)
#include <emmintrin.h>
#endif

#include "pmb200.h"
#include "pmb200_peer.h"
#include "pm_layout.h"
#include "pm_capi.h"
#include "host_pool.h"

namespace pm {
int launch_analyze(const pm_trials& T, const pm_policy& P, const pm_trial_results& R, int max_covering,
                   double* gscratch, cudaStream_t stream, size_t* scratch_bytes_needed,
                   const pm_peer_rows* rows = nullptr);
int launch_bootstrap(const BootArgs& A, cudaStream_t stream, const pm_peer_groups* groups = nullptr);
int launch_bootstrap_prepare(const BootArgs& A, cudaStream_t stream);
int launch_resample_indices(uint64_t seed, int n, int B, int32_t* out, cudaStream_t stream);
int prepare_bootstrap_constants(int device);

static thread_local std::string t_error;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap; va_start(ap, fmt); vsnprintf(buf, sizeof buf, fmt, ap); va_end(ap);
  t_error = buf;
  return code;
}
int cuda_fail(cudaError_t e, const char* where) {
  return fail(PM_E_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

Arena g_arenas[kMaxDevices];

int check_bootstrap_fits(int n_metrics, int max_members) {
  size_t available = 0;
  const size_t need = bootstrap_smem_shortfall(n_metrics, max_members, &available);
  if (need)
    return fail(PM_E_LIMIT, "bootstrap of %d metrics with groups of up to %d members needs %zu bytes of shared memory per "
                "block; the device offers %zu", n_metrics, max_members, need, available);
  return PM_OK;
}

int current_device(int* device) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) { cudaGetLastError(); return fail(PM_E_NODEVICE, "no CUDA device visible (%s)", cudaGetErrorString(e)); }
  e = cudaGetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*device < 0 || *device >= kMaxDevices) return fail(PM_E_LIMIT, "device ordinal %d beyond %d", *device, kMaxDevices);
  return PM_OK;
}

int arena_reserve(Arena& a, size_t dev_bytes, size_t host_bytes) {
  if (dev_bytes > a.dev_bytes) {
    if (a.dev) cudaFree(a.dev);
    a.dev = nullptr; a.dev_bytes = 0;
    cudaError_t e = cudaMalloc(&a.dev, dev_bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(workspace)");
    a.dev_bytes = dev_bytes;
  }
  if (host_bytes > a.host_bytes) {
    if (a.host) cudaFreeHost(a.host);
    a.host = nullptr; a.host_bytes = 0;
    cudaError_t e = cudaMallocHost(&a.host, host_bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocHost(staging)");
    a.host_bytes = host_bytes;
  }
  if (!a.stream) {
    cudaError_t e = cudaStreamCreateWithFlags(&a.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
  }
  if (!a.side) {
    cudaError_t e = cudaStreamCreateWithFlags(&a.side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a.join, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a.analysed, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a.results, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "side stream / events");
  }
  return PM_OK;
}

namespace {

// Visit every array of a pm_trials batch with its element count, in one
// fixed order shared by the sizing and the staging passes.
template <class T, class F> void visit_trials(T& t, F f) {
  const size_t nt = (size_t)t.n_trials, ns = (size_t)t.n_samples, ne = (size_t)t.n_epochs;
  // A broadcast column holds one element for every sample.
  auto per = [&](uint32_t bit) { return (t.broadcast_columns & bit) ? (ns ? size_t(1) : size_t(0)) : ns; };
  f(t.phase_offsets, nt * PM_PHASES + 1);
  f(t.phase_start_s, nt * PM_PHASES); f(t.phase_end_s, nt * PM_PHASES); f(t.phase_present, nt * PM_PHASES);
  f(t.t_s, ns); f(t.power_w, per(PM_COL_POWER_W)); f(t.memory_power_w, per(PM_COL_MEMORY_POWER_W));
  f(t.graphics_clock_mhz, per(PM_COL_GRAPHICS_CLOCK)); f(t.sm_clock_mhz, per(PM_COL_SM_CLOCK));
  f(t.memory_clock_mhz, per(PM_COL_MEMORY_CLOCK)); f(t.temperature_c, per(PM_COL_TEMPERATURE));
  f(t.power_limit_w, per(PM_COL_POWER_LIMIT)); f(t.enforced_power_limit_w, per(PM_COL_ENFORCED_LIMIT));
  f(t.pstate, per(PM_COL_PSTATE));
  f(t.energy_int, per(PM_COL_ENERGY_INT)); f(t.energy_float, per(PM_COL_ENERGY_FLOAT));
  f(t.throttle_reasons, per(PM_COL_THROTTLE)); f(t.sample_flags, per(PM_COL_SAMPLE_FLAGS));
  f(t.memory_power_source, per(PM_COL_MEMORY_SOURCE));
  f(t.epoch_offsets, nt * 2 + 1); f(t.epoch_status, nt * 2);
  f(t.epoch_start_s, ne); f(t.epoch_end_s, ne); f(t.epoch_operations, ne); f(t.epoch_logical_bytes, ne);
  f(t.epoch_loop_slots, ne); f(t.epoch_counts_exact, ne);
  f(t.trial_scalars, nt * PM_TS_COUNT); f(t.trial_flags, nt);
}

constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Structural checks of a host batch (sizes, NULL arrays, offsets, limits).
// The per-sample order check runs in the staging pass (scan_slots).
int check_trials_host(const pm_trials& T) {
  if (T.n_trials < 0 || T.n_samples < 0 || T.n_epochs < 0) return fail(PM_E_INVALID, "negative batch size");
  if (T.broadcast_columns & ~uint32_t(PM_COL_ALL)) return fail(PM_E_INVALID, "broadcast_columns has unknown bits");
  bool null_seen = false;
  visit_trials(T, [&](const auto* p, size_t n) { if (n && !p) null_seen = true; });
  if (null_seen) return fail(PM_E_INVALID, "a pm_trials array is NULL");
  if (T.phase_offsets[0] != 0 || T.phase_offsets[(size_t)T.n_trials * PM_PHASES] != T.n_samples)
    return fail(PM_E_INVALID, "phase_offsets must start at 0 and end at n_samples");
  for (size_t s = 0; s < (size_t)T.n_trials * PM_PHASES; ++s) {
    const int64_t b = T.phase_offsets[s], e = T.phase_offsets[s + 1];
    if (e < b) return fail(PM_E_INVALID, "phase_offsets must be non-decreasing");
    if (e - b > kMaxPhaseSamples) return fail(PM_E_LIMIT, "a phase holds %lld samples; the limit is %d", (long long)(e - b), kMaxPhaseSamples);
  }
  if (T.epoch_offsets[0] != 0 || T.epoch_offsets[(size_t)T.n_trials * 2] != T.n_epochs)
    return fail(PM_E_INVALID, "epoch_offsets must start at 0 and end at n_epochs");
  for (size_t s = 0; s < (size_t)T.n_trials * 2; ++s) {
    const int32_t n = T.epoch_offsets[s + 1] - T.epoch_offsets[s];
    if (n < 0) return fail(PM_E_INVALID, "epoch_offsets must be non-decreasing");
    if (n > kMaxEpochsPerArm) return fail(PM_E_LIMIT, "an arm lists %d epochs; the limit is %d", n, kMaxEpochsPerArm);
  }
  return PM_OK;
}

// Phase slots [s0, s1): the longest phase, and the first slot whose t_s does
// not increase strictly (-1 if none).
void scan_slots(const pm_trials& T, size_t s0, size_t s1, int64_t* longest, int64_t* bad_slot) {
  int64_t mc = 0, bad = -1;
  for (size_t s = s0; s < s1 && bad < 0; ++s) {
    const int64_t b = T.phase_offsets[s], e = T.phase_offsets[s + 1];
    for (int64_t i = b + 1; i < e; ++i)
      if (!(T.t_s[i] > T.t_s[i - 1])) { bad = (int64_t)s; break; }
    if (e - b > mc) mc = e - b;
  }
  *longest = mc;
  *bad_slot = bad;
}

template <class F> void visit_results(pm_trial_results& r, size_t n, F f) {
  f(r.phase_out, n * PM_PHASES * PM_PO_COUNT); f(r.phase_flags, n * PM_PHASES); f(r.trial_out, n * PM_TO_COUNT);
  f(r.issue_bits, n * PM_ISSUE_WORDS); f(r.metrics, n * PM_N_METRICS); f(r.valid, n);
}

// Lay out arrays back to back (256-byte aligned) starting at `base`.
struct Layout {
  char* base; size_t used = 0;
  template <class P> void place(P*& p, size_t count) {
    used = align256(used);
    p = reinterpret_cast<P*>(base + used);
    used += count * sizeof(P);
  }
};

// memcpy into the pinned staging buffer with non-temporal stores: the lines
// go to memory instead of this core's cache, so the DMA that reads them next
// does not have to fetch them back out of other cores' caches, and no line
// is read for ownership first.  `dst` is 16-byte aligned (arena offsets are).
void stream_copy(char* dst, const char* src, size_t bytes) {
#if defined(__x86_64__)
  size_t i = 0;
  if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    for (; i + 64 <= bytes; i += 64) {
      const __m128i a = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i));
      const __m128i b = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i + 16));
      const __m128i c = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i + 32));
      const __m128i d = _mm_loadu_si128(reinterpret_cast<const __m128i*>(src + i + 48));
      _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i), a);
      _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i + 16), b);
      _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i + 32), c);
      _mm_stream_si128(reinterpret_cast<__m128i*>(dst + i + 48), d);
    }
    _mm_sfence();   // the streamed lines are visible before the task reports done
  }
  if (i < bytes) memcpy(dst + i, src + i, bytes - i);
#else
  memcpy(dst, src, bytes);
#endif
}

}  // namespace

size_t analyze_scratch_bytes(int n_trials, int max_phase_samples) {
  int SP = 32;
  while (SP < max_phase_samples + 1) SP <<= 1;
  const size_t tile = (size_t)kSortColumns * SP * sizeof(double);
  return tile > kSmemSortBytes ? (size_t)n_trials * tile : 0;
}

}  // namespace pm

using namespace pm;

extern "C" {

size_t pm_last_error(char* buffer, size_t cap) {
  if (buffer && cap) {
    const size_t n = t_error.size() < cap - 1 ? t_error.size() : cap - 1;
    memcpy(buffer, t_error.data(), n);
    buffer[n] = 0;
  }
  return t_error.size();
}

int32_t pm_abi_version(void) { return PM_ABI_VERSION; }

int32_t pm_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
  return n;
}

int32_t pm_layout(const char* name) {
  if (!name) return -1;
#define PM_LOOKUP(list)                                                     \
  {                                                                         \
    static const char* names[] = {list};                                    \
    for (int i = 0; i < (int)(sizeof(names) / sizeof(names[0])); ++i)       \
      if (!strcmp(name, names[i])) return i;                                \
  }
#define PM_NAME_PO(n) "PM_PO_" #n,
#define PM_NAME_PF(n) "PM_PF_" #n,
#define PM_NAME_TO(n) "PM_TO_" #n,
#define PM_NAME_IT(n) "PM_IT_" #n,
#define PM_NAME_IB(n) "PM_IB_" #n,
#define PM_NAME_IP(n) "PM_IP_" #n,
#define PM_NAME_W(n) "PM_W_" #n,
#define PM_NAME_M(n) "PM_M_" #n,
  PM_LOOKUP(PM_PHASE_FIELDS(PM_NAME_PO))
  PM_LOOKUP(PM_PHASE_FLAGS(PM_NAME_PF))
  PM_LOOKUP(PM_TRIAL_FIELDS(PM_NAME_TO))
  PM_LOOKUP(PM_ISSUES_TREATMENT(PM_NAME_IT))
  PM_LOOKUP(PM_ISSUES_BASELINE(PM_NAME_IB))
  PM_LOOKUP(PM_ISSUES_PAIRED(PM_NAME_IP))
  PM_LOOKUP(PM_WARNINGS(PM_NAME_W))
  PM_LOOKUP(PM_METRIC_NAMES(PM_NAME_M))
  static const struct { const char* n; int v; } counts[] = {
    {"PM_PO_COUNT", PM_PO_COUNT}, {"PM_PF_COUNT", PM_PF_COUNT}, {"PM_TO_COUNT", PM_TO_COUNT},
    {"PM_IT_COUNT", PM_IT_COUNT}, {"PM_IB_COUNT", PM_IB_COUNT}, {"PM_IP_COUNT", PM_IP_COUNT},
    {"PM_W_COUNT", PM_W_COUNT}, {"PM_M_COUNT", PM_M_COUNT}, {"PM_ISSUE_WORDS", PM_ISSUE_WORDS},
    {"PM_TS_COUNT", PM_TS_COUNT}, {"PM_PHASES", PM_PHASES},
    {"PM_MAX_PHASE_SAMPLES", kMaxPhaseSamples}, {"PM_MAX_EPOCHS_PER_ARM", kMaxEpochsPerArm},
    {"PM_MAX_GROUP_MEMBERS", kMaxGroupMembers}};
  for (auto& c : counts) if (!strcmp(name, c.n)) return c.v;
  return -1;
}

size_t pm_analyze_scratch_bytes(int32_t n_trials, int32_t max_phase_samples) {
  return analyze_scratch_bytes(n_trials < 0 ? 0 : n_trials, max_phase_samples < 0 ? 0 : max_phase_samples);
}

int pm_analyze_trials_device(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out,
                             void* scratch, size_t scratch_bytes, void* stream) {
  if (!trials || !policy || !out) return fail(PM_E_INVALID, "NULL argument");
  if (trials->n_trials < 0 || trials->max_phase_samples < 0) return fail(PM_E_INVALID, "negative size");
  if (trials->broadcast_columns & ~uint32_t(PM_COL_ALL)) return fail(PM_E_INVALID, "broadcast_columns has unknown bits");
  if (trials->max_phase_samples > kMaxPhaseSamples) return fail(PM_E_LIMIT, "max_phase_samples beyond %d", kMaxPhaseSamples);
  if (policy->min_samples < 2) return fail(PM_E_INVALID, "min_samples must be >= 2");
  const size_t need = analyze_scratch_bytes(trials->n_trials, trials->max_phase_samples);
  if (need > scratch_bytes || (need && !scratch))
    return fail(PM_E_INVALID, "analysis needs %zu bytes of device scratch, got %zu", need, scratch_bytes);
  if (need && reinterpret_cast<uintptr_t>(scratch) % 16)
    return fail(PM_E_INVALID, "the analysis's device scratch must be 16-byte aligned");
  launch_analyze(*trials, *policy, *out, trials->max_phase_samples, need ? (double*)scratch : nullptr, (cudaStream_t)stream, nullptr);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "analyze_kernel launch");
  return PM_OK;
}

int pm_analyze_trials_device_exchange(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out,
                                      void* scratch, size_t scratch_bytes, const pm_peer_rows* rows, void* stream) {
  if (!rows) return fail(PM_E_INVALID, "NULL rows");
  if (rows->n_ranks < 1 || rows->n_ranks > PM_MAX_RANKS || rows->rank < 0 || rows->rank >= rows->n_ranks)
    return fail(PM_E_INVALID, "bad rank geometry");
  if (rows->row_offset < 0 || rows->epoch == 0 || !rows->done) return fail(PM_E_INVALID, "bad row offset, epoch or counter");
  for (int r = 0; r < rows->n_ranks; ++r)
    if (!rows->metrics[r] || !rows->valid[r] || !rows->flags[r]) return fail(PM_E_INVALID, "a rank's buffer is NULL");
  if (!trials || !policy || !out) return fail(PM_E_INVALID, "NULL argument");
  if (trials->n_trials < 0 || trials->max_phase_samples < 0) return fail(PM_E_INVALID, "negative size");
  if (trials->broadcast_columns & ~uint32_t(PM_COL_ALL)) return fail(PM_E_INVALID, "broadcast_columns has unknown bits");
  if (trials->max_phase_samples > kMaxPhaseSamples) return fail(PM_E_LIMIT, "max_phase_samples beyond %d", kMaxPhaseSamples);
  if (policy->min_samples < 2) return fail(PM_E_INVALID, "min_samples must be >= 2");
  const size_t need = analyze_scratch_bytes(trials->n_trials, trials->max_phase_samples);
  if (need > scratch_bytes || (need && !scratch))
    return fail(PM_E_INVALID, "analysis needs %zu bytes of device scratch, got %zu", need, scratch_bytes);
  if (need && reinterpret_cast<uintptr_t>(scratch) % 16)
    return fail(PM_E_INVALID, "the analysis's device scratch must be 16-byte aligned");
  launch_analyze(*trials, *policy, *out, trials->max_phase_samples, need ? (double*)scratch : nullptr, (cudaStream_t)stream,
                 nullptr, rows);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "analyze_kernel launch");
  return PM_OK;
}

}  // extern "C"

namespace pm {
namespace {

struct StagedTrials {
  pm_trials dev;              // device view of the staged batch
  pm_trial_results dres, hres;
  size_t in_bytes = 0, res_bytes = 0, end = 0;   // byte extents inside the arena
  size_t scratch = 0;         // analysis scratch (long phases), after the caller's extra device bytes
  int max_cov = 0;
  double* gscratch = nullptr;
};

// Check a host batch and size its arena layout: inputs, then results, then
// (after the caller's extra device bytes) the analysis scratch.
int plan_trials(const pm_trials& T, StagedTrials& S) {
  int rc = check_trials_host(T);
  if (rc) return rc;
  const size_t n = (size_t)T.n_trials;
  visit_trials(T, [&](const auto* p, size_t count) { S.in_bytes = align256(S.in_bytes) + count * sizeof(*p); });
  S.in_bytes = align256(S.in_bytes);
  pm_trial_results probe{};
  visit_results(probe, n, [&](auto* p, size_t count) { S.res_bytes = align256(S.res_bytes) + count * sizeof(*p); });
  S.res_bytes = align256(S.res_bytes);
  // The scratch size depends on the longest phase, known only after the scan:
  // reserve for the worst case the batch allows (its longest offsets span).
  int64_t bound = 0;
  for (size_t s = 0; s < n * PM_PHASES; ++s) bound = std::max<int64_t>(bound, T.phase_offsets[s + 1] - T.phase_offsets[s]);
  S.scratch = analyze_scratch_bytes((int)n, (int)bound);
  S.end = S.in_bytes + S.res_bytes;
  S.max_cov = (int)bound;
  return PM_OK;
}

// Stage a planned batch into the reserved arena and enqueue its H2D copy on
// A.stream; points S.dev's arrays into the arena.
int copy_trials(Arena& A, const pm_trials& T, StagedTrials& S) {
  const size_t n = (size_t)T.n_trials;
  S.dev = T;
  S.dev.max_phase_samples = S.max_cov;
  // Copy pieces of at most kPiece bytes in destination order, then the
  // sample-order scan in slot ranges; pool threads and this thread share them.
  // Small pieces make the staged prefix grow steadily, so its DMA (issued a
  // kDma chunk at a time: on B200 1 MiB copies reach 43 GB/s where one 3.4 MB
  // copy reached 20) runs alongside the staging instead of after it.
  constexpr size_t kPiece = size_t(128) << 10, kDma = size_t(1) << 20;
  struct Piece { const char* src; size_t dst; size_t bytes; };
  std::vector<Piece> pieces;
  pieces.reserve(S.in_bytes / kPiece + 64);
  Layout hl{static_cast<char*>(A.host)};
  size_t offs[32]; int k = 0;
  visit_trials(T, [&](const auto* p, size_t count) {
    using E = std::remove_cv_t<std::remove_pointer_t<decltype(p)>>;
    E* dst = nullptr;
    hl.place(dst, count);
    const size_t at = reinterpret_cast<char*>(dst) - static_cast<char*>(A.host);
    const size_t bytes = count * sizeof(E);
    for (size_t o = 0; o < bytes; o += kPiece)
      pieces.push_back({reinterpret_cast<const char*>(p) + o, at + o, std::min(kPiece, bytes - o)});
    offs[k++] = at;
  });
  const size_t slots = n * PM_PHASES;
  const size_t scan_tasks = slots ? std::min<size_t>(64, (slots + 255) / 256) : 0;
  std::vector<int64_t> longest(scan_tasks, 0), bad(scan_tasks, -1);
  char* host = static_cast<char*>(A.host);
  char* dev = static_cast<char*>(A.dev);
  HostBatch batch(pieces.size() + scan_tasks, [&](size_t i) {
    if (i < pieces.size()) {
      stream_copy(host + pieces[i].dst, pieces[i].src, pieces[i].bytes);
    } else {
      const size_t t = i - pieces.size();
      scan_slots(T, slots * t / scan_tasks, slots * (t + 1) / scan_tasks, &longest[t], &bad[t]);
    }
  });
  // Start the DMA of the contiguous staged prefix a chunk at a time as soon
  // as it is complete (the last chunk may be shorter).
  size_t ready = 0, issued = 0;
  cudaError_t dma = cudaSuccess;
  auto progress = [&] {
    while (ready < pieces.size() && batch.done(ready)) ++ready;
    const bool all = ready == pieces.size();
    const size_t upto = all ? S.in_bytes : (ready ? pieces[ready - 1].dst + pieces[ready - 1].bytes : 0);
    while (dma == cudaSuccess && upto > issued && (upto - issued >= kDma || all)) {
      const size_t bytes = std::min(kDma, upto - issued);
      dma = cudaMemcpyAsync(dev + issued, host + issued, bytes, cudaMemcpyHostToDevice, A.stream);
      issued += bytes;
    }
  };
  run_host_batch(batch, progress);
  progress();
  if (dma != cudaSuccess) {
    cudaStreamSynchronize(A.stream);
    return cuda_fail(dma, "cudaMemcpyAsync(inputs)");
  }
  for (size_t t = 0; t < scan_tasks; ++t) {
    if (bad[t] >= 0) {
      cudaStreamSynchronize(A.stream);   // the staged copy must finish before the buffer is reused
      return fail(PM_E_INVALID, "t_s must increase strictly within a phase (slot %lld)", (long long)bad[t]);
    }
  }
  k = 0;
  visit_trials(S.dev, [&](auto& p, size_t) {
    using Ptr = std::remove_reference_t<decltype(p)>;
    p = reinterpret_cast<Ptr>(dev + offs[k++]);
  });
  return PM_OK;
}

// Point S.dres, S.hres and S.gscratch into a reserved arena.
void place_results(Arena& A, size_t n, size_t extra_dev, StagedTrials& S) {
  char* dev = static_cast<char*>(A.dev);
  Layout dl{dev + S.in_bytes}, rl{static_cast<char*>(A.host) + S.in_bytes};
  visit_results(S.dres, n, [&](auto*& p, size_t count) { dl.place(p, count); });
  visit_results(S.hres, n, [&](auto*& p, size_t count) { rl.place(p, count); });
  S.gscratch = S.scratch ? reinterpret_cast<double*>(dev + S.end + extra_dev) : nullptr;
}

// plan_trials, arena_reserve (plus `extra_dev`/`extra_host` bytes after the
// results) and copy_trials in one step.
int stage_trials(Arena& A, const pm_trials& T, size_t extra_dev, size_t extra_host, StagedTrials& S) {
  int rc = plan_trials(T, S);
  if (rc) return rc;
  if ((rc = arena_reserve(A, S.end + S.scratch + extra_dev, S.end + extra_host))) return rc;
  place_results(A, (size_t)T.n_trials, extra_dev, S);
  return copy_trials(A, T, S);
}

// Copy the pinned results into the caller's arrays (those not NULL), in
// 64 KiB pieces shared by the host pool and this thread.
void copy_results_out(const StagedTrials& S, size_t n, pm_trial_results* out) {
  struct Piece { char* dst; const char* src; size_t bytes; };
  std::vector<Piece> pieces;
  auto add = [&](void* dst, const void* src, size_t bytes) {
    constexpr size_t kPiece = size_t(64) << 10;
    if (!dst) return;
    for (size_t o = 0; o < bytes; o += kPiece)
      pieces.push_back({static_cast<char*>(dst) + o, static_cast<const char*>(src) + o, std::min(kPiece, bytes - o)});
  };
  add(out->phase_out, S.hres.phase_out, n * PM_PHASES * PM_PO_COUNT * sizeof(double));
  add(out->phase_flags, S.hres.phase_flags, n * PM_PHASES * sizeof(uint32_t));
  add(out->trial_out, S.hres.trial_out, n * PM_TO_COUNT * sizeof(double));
  add(out->issue_bits, S.hres.issue_bits, n * PM_ISSUE_WORDS * sizeof(uint64_t));
  add(out->metrics, S.hres.metrics, n * PM_N_METRICS * sizeof(double));
  add(out->valid, S.hres.valid, n);
  HostBatch batch(pieces.size(), [&](size_t i) { memcpy(pieces[i].dst, pieces[i].src, pieces[i].bytes); });
  run_host_batch(batch, nullptr);
}

}  // namespace
}  // namespace pm

// ---------------------------------------------------------------------------
// Shared by every bootstrap entry point (the allocation-free one included).
int pm::check_bootstrap(const pm_bootstrap_job* j) {
  if (!j) return fail(PM_E_INVALID, "NULL job");
  if (j->n_groups < 0 || j->n_metrics <= 0 || j->n_metrics > kMaxMetrics || j->n_members < 0 || j->n_rows < 0)
    return fail(PM_E_INVALID, "bad bootstrap sizes");
  if (j->resamples < 40 || j->resamples > (1 << 24)) return fail(PM_E_INVALID, "resamples must be in [40, 2^24]");
  if (j->max_members < 0 || j->max_members > kMaxGroupMembers)
    return fail(PM_E_LIMIT, "max_members %d outside [0, %d]", j->max_members, kMaxGroupMembers);
  if (!j->values || !j->group_offsets || !j->seeds || !j->medians || !j->ci_lo || !j->ci_hi)
    return fail(PM_E_INVALID, "a pm_bootstrap_job array is NULL");
  return PM_OK;
}

extern "C" {

int pm_analyze_trials(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out) {
  if (!trials || !policy || !out) return fail(PM_E_INVALID, "NULL argument");
  int device = 0, rc = current_device(&device);
  if (rc) return rc;
  if (policy->min_samples < 2) return fail(PM_E_INVALID, "min_samples must be >= 2");
  const size_t n = (size_t)trials->n_trials;
  if (trials->n_trials < 0) return fail(PM_E_INVALID, "negative n_trials");
  if (n == 0) return PM_OK;
  Arena& A = g_arenas[device];
  std::lock_guard<std::mutex> guard(A.lock);
  StagedTrials S;
  if ((rc = stage_trials(A, *trials, 0, 0, S))) return rc;
  launch_analyze(S.dev, *policy, S.dres, S.max_cov, S.gscratch, A.stream, nullptr);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "analyze_kernel launch");
  e = cudaMemcpyAsync(static_cast<char*>(A.host) + S.in_bytes, static_cast<char*>(A.dev) + S.in_bytes, S.res_bytes,
                      cudaMemcpyDeviceToHost, A.stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(results)");
  e = cudaStreamSynchronize(A.stream);
  if (e != cudaSuccess) return cuda_fail(e, "analyze_kernel");
  copy_results_out(S, n, out);
  return PM_OK;
}

size_t pm_bootstrap_scratch_bytes(int32_t n_groups, int32_t max_members, int32_t resamples) {
  if (n_groups < 0 || max_members < 0 || resamples < 0) return 0;
  return bootstrap_scratch_bytes(n_groups, max_members, resamples);
}

// Shared by the device bootstrap entry points: checks and the kernel arguments.
static int device_boot_args(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes, BootArgs* out) {
  int rc = check_bootstrap(job);
  if (rc) return rc;
  if (reinterpret_cast<uintptr_t>(scratch) % 16)
    return fail(PM_E_INVALID, "the bootstrap's device scratch must be 16-byte aligned");
  int device = 0;
  if ((rc = current_device(&device))) return rc;
  if (prepare_bootstrap_constants(device)) return fail(PM_E_CUDA, "bootstrap constants upload failed");
  if ((rc = check_bootstrap_fits(job->n_metrics, job->max_members))) return rc;
  // pm_bootstrap_scratch_bytes sizes the streamed layout; a scratch holding only
  // the histograms (and the streams of groups above seven members) still works,
  // with the draws consumed as they are generated.
  const bool streamed = scratch && bootstrap_scratch_bytes(job->n_groups, job->max_members, job->resamples) <= scratch_bytes;
  const size_t need = bootstrap_scratch_bytes(job->n_groups, job->max_members, job->resamples, streamed);
  if (need > scratch_bytes || (need && !scratch))
    return fail(PM_E_INVALID, "bootstrap needs %zu bytes of device scratch, got %zu", need, scratch_bytes);
  *out = BootArgs{job->n_groups, job->n_metrics, job->resamples, job->max_members, job->values, job->group_offsets,
                  job->member_rows, job->member_valid, job->seeds, job->medians, job->ci_lo, job->ci_hi,
                  static_cast<uint8_t*>(scratch), 1, streamed ? 1 : 0};
  return PM_OK;
}

int pm_bootstrap_prepare_device(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes, void* stream) {
  BootArgs A;
  int rc = device_boot_args(job, scratch, scratch_bytes, &A);
  if (rc) return rc;
  launch_bootstrap_prepare(A, (cudaStream_t)stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_prepare_kernel launch");
  return PM_OK;
}

int pm_bootstrap_finish_device(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes, void* stream) {
  BootArgs A;
  int rc = device_boot_args(job, scratch, scratch_bytes, &A);
  if (rc) return rc;
  launch_bootstrap(A, (cudaStream_t)stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_kernel launch");
  return PM_OK;
}

int pm_bootstrap_finish_device_exchange(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes,
                                        const pm_peer_groups* groups, void* stream) {
  if (!groups) return fail(PM_E_INVALID, "NULL groups");
  if (groups->n_ranks < 1 || groups->n_ranks > PM_MAX_RANKS || groups->rank < 0 || groups->rank >= groups->n_ranks)
    return fail(PM_E_INVALID, "bad rank geometry");
  if (groups->root < -1 || groups->root >= groups->n_ranks) return fail(PM_E_INVALID, "root must be -1 or a rank");
  if (groups->epoch == 0 || !groups->done) return fail(PM_E_INVALID, "bad epoch or counter");
  for (int r = 0; r < groups->n_ranks; ++r)
    if ((groups->root < 0 || r == groups->root) && (!groups->out[r] || !groups->flags[r]))
      return fail(PM_E_INVALID, "a receiving rank's buffer is NULL");
  BootArgs A;
  int rc = device_boot_args(job, scratch, scratch_bytes, &A);
  if (rc) return rc;
  if (groups->per_rank < A.n_groups) return fail(PM_E_INVALID, "per_rank below this rank's group count");
  launch_bootstrap(A, (cudaStream_t)stream, groups);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_kernel launch");
  return PM_OK;
}

// The device sweep's own side stream and fork/join events, one set per device
// (created on first use with that device current); the mutex keeps one call's
// record/wait pairs together when several host threads call at once.
struct SweepFork {
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex lock;
};
static SweepFork g_sweep_fork[kMaxDevices];

size_t pm_analyze_sweep_scratch_bytes(int32_t n_trials, int32_t max_phase_samples, int32_t n_groups,
                                      int32_t max_members, int32_t resamples) {
  if (n_trials < 0 || max_phase_samples < 0 || n_groups < 0 || max_members < 0 || resamples < 0) return 0;
  return align256(analyze_scratch_bytes(n_trials, max_phase_samples)) +
         bootstrap_scratch_bytes(n_groups, max_members, resamples);
}

int pm_analyze_sweep_device(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out,
                            const pm_bootstrap_job* groups, void* scratch, size_t scratch_bytes,
                            const pm_peer_groups* exchange, void* stream) {
  if (!trials || !policy || !out || !groups) return fail(PM_E_INVALID, "NULL argument");
  if (trials->n_trials < 0 || trials->max_phase_samples < 0) return fail(PM_E_INVALID, "negative size");
  if (trials->broadcast_columns & ~uint32_t(PM_COL_ALL)) return fail(PM_E_INVALID, "broadcast_columns has unknown bits");
  if (trials->max_phase_samples > kMaxPhaseSamples) return fail(PM_E_LIMIT, "max_phase_samples beyond %d", kMaxPhaseSamples);
  if (policy->min_samples < 2) return fail(PM_E_INVALID, "min_samples must be >= 2");
  if (exchange) {
    if (exchange->n_ranks < 1 || exchange->n_ranks > PM_MAX_RANKS || exchange->rank < 0 || exchange->rank >= exchange->n_ranks)
      return fail(PM_E_INVALID, "bad rank geometry");
    if (exchange->root < -1 || exchange->root >= exchange->n_ranks) return fail(PM_E_INVALID, "root must be -1 or a rank");
    if (exchange->epoch == 0 || !exchange->done) return fail(PM_E_INVALID, "bad epoch or counter");
    for (int r = 0; r < exchange->n_ranks; ++r)
      if ((exchange->root < 0 || r == exchange->root) && (!exchange->out[r] || !exchange->flags[r]))
        return fail(PM_E_INVALID, "a receiving rank's buffer is NULL");
    if (exchange->per_rank < groups->n_groups) return fail(PM_E_INVALID, "per_rank below this rank's group count");
  }
  const size_t a_need = analyze_scratch_bytes(trials->n_trials, trials->max_phase_samples);
  const size_t b_off = align256(a_need);
  const size_t b_need = bootstrap_scratch_bytes(groups->n_groups, groups->max_members, groups->resamples);
  if (b_off + b_need > scratch_bytes || (b_off + b_need > 0 && !scratch))
    return fail(PM_E_INVALID, "the sweep needs %zu bytes of device scratch (pm_analyze_sweep_scratch_bytes), got %zu",
                b_off + b_need, scratch_bytes);
  if (reinterpret_cast<uintptr_t>(scratch) % 256)
    return fail(PM_E_INVALID, "the sweep's device scratch must be 256-byte aligned");
  BootArgs A;
  int rc = device_boot_args(groups, static_cast<uint8_t*>(scratch) + b_off, scratch_bytes - b_off, &A);
  if (rc) return rc;
  int device = 0;
  if ((rc = current_device(&device))) return rc;
  SweepFork& F = g_sweep_fork[device];
  std::lock_guard<std::mutex> guard(F.lock);
  if (!F.side) {
    cudaError_t e = cudaStreamCreateWithFlags(&F.side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&F.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&F.join, cudaEventDisableTiming);
    if (e != cudaSuccess) { F.side = nullptr; return cuda_fail(e, "sweep side stream / events"); }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The draws need only the seeds and group sizes: on the side stream, beside
  // the analysis on the caller's stream (one CTA per trial), joined before the
  // finish.
  cudaError_t e = cudaEventRecord(F.fork, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(F.side, F.fork, 0);
  if (e != cudaSuccess) return cuda_fail(e, "sweep fork");
  launch_bootstrap_prepare(A, F.side);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_prepare_kernel launch");
  e = cudaEventRecord(F.join, F.side);
  if (e != cudaSuccess) return cuda_fail(e, "sweep join record");
  launch_analyze(*trials, *policy, *out, trials->max_phase_samples, a_need ? static_cast<double*>(scratch) : nullptr, s,
                 nullptr);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "analysis launch");
  e = cudaStreamWaitEvent(s, F.join, 0);
  if (e != cudaSuccess) return cuda_fail(e, "sweep join");
  launch_bootstrap(A, s, exchange);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_kernel launch");
  return PM_OK;
}

int pm_group_bootstrap_device(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes, void* stream) {
  int rc = pm_bootstrap_prepare_device(job, scratch, scratch_bytes, stream);
  return rc ? rc : pm_bootstrap_finish_device(job, scratch, scratch_bytes, stream);
}

int pm_group_bootstrap(const pm_bootstrap_job* job) {
  int rc = check_bootstrap(job);
  if (rc) return rc;
  int device = 0;
  if ((rc = current_device(&device))) return rc;
  if (prepare_bootstrap_constants(device)) return fail(PM_E_CUDA, "bootstrap constants upload failed");
  const size_t G = (size_t)job->n_groups, M = (size_t)job->n_metrics;
  int mm = 0;
  for (size_t g = 0; g < G; ++g) {
    const int c = job->group_offsets[g + 1] - job->group_offsets[g];
    if (c < 0) return fail(PM_E_INVALID, "group_offsets must be non-decreasing");
    if (c > kMaxGroupMembers) return fail(PM_E_LIMIT, "group %zu lists %d members; the limit is %d", g, c, kMaxGroupMembers);
    if (c > mm) mm = c;
  }
  if (G && (job->group_offsets[0] != 0 || job->group_offsets[G] != job->n_members))
    return fail(PM_E_INVALID, "group_offsets must start at 0 and end at n_members");
  const size_t rows = job->member_rows || job->member_valid ? (size_t)job->n_rows : (size_t)job->n_members;
  if (job->member_rows)
    for (int i = 0; i < job->n_members; ++i)
      if (job->member_rows[i] < 0 || (size_t)job->member_rows[i] >= rows) return fail(PM_E_INVALID, "member_rows[%d] out of range", i);
  if (G == 0) return PM_OK;
  if ((rc = check_bootstrap_fits((int)M, mm))) return rc;
  const size_t scratch = bootstrap_scratch_bytes((int)G, mm, job->resamples);
  size_t in_bytes = align256(rows * M * 8) + align256((G + 1) * 4) + align256((size_t)job->n_members * 4) + align256(rows) + align256(G * 8);
  size_t out_bytes = 3 * align256(G * M * 8);
  Arena& A = g_arenas[device];
  std::lock_guard<std::mutex> guard(A.lock);
  if ((rc = arena_reserve(A, in_bytes + out_bytes + scratch, in_bytes + out_bytes))) return rc;
  Layout hl{static_cast<char*>(A.host)};
  double* hv; int32_t* ho; int32_t* hr = nullptr; uint8_t* hvalid = nullptr; uint64_t* hs;
  hl.place(hv, rows * M); memcpy(hv, job->values, rows * M * 8);
  hl.place(ho, G + 1); memcpy(ho, job->group_offsets, (G + 1) * 4);
  int32_t* tmp_r; hl.place(tmp_r, job->n_members); if (job->member_rows) { memcpy(tmp_r, job->member_rows, (size_t)job->n_members * 4); hr = tmp_r; }
  uint8_t* tmp_v; hl.place(tmp_v, rows); if (job->member_valid) { memcpy(tmp_v, job->member_valid, rows); hvalid = tmp_v; }
  hl.place(hs, G); memcpy(hs, job->seeds, G * 8);
  auto dev_of = [&](const void* h) { return static_cast<char*>(A.dev) + (static_cast<const char*>(h) - static_cast<char*>(A.host)); };
  cudaStream_t st = A.stream;
  cudaError_t e = cudaMemcpyAsync(A.dev, A.host, in_bytes, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(bootstrap inputs)");
  char* dout = static_cast<char*>(A.dev) + in_bytes;
  double* dmed = reinterpret_cast<double*>(dout);
  double* dlo = reinterpret_cast<double*>(dout + align256(G * M * 8));
  double* dhi = reinterpret_cast<double*>(dout + 2 * align256(G * M * 8));
  BootArgs args{(int)G, (int)M, job->resamples, mm, reinterpret_cast<const double*>(dev_of(hv)),
                reinterpret_cast<const int32_t*>(dev_of(ho)), hr ? reinterpret_cast<const int32_t*>(dev_of(hr)) : nullptr,
                hvalid ? reinterpret_cast<const uint8_t*>(dev_of(hvalid)) : nullptr,
                reinterpret_cast<const uint64_t*>(dev_of(hs)), dmed, dlo, dhi,
                reinterpret_cast<uint8_t*>(dout + out_bytes), 1, 1};
  launch_bootstrap_prepare(args, st);
  launch_bootstrap(args, st);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_kernel launch");
  char* hout = static_cast<char*>(A.host) + in_bytes;
  e = cudaMemcpyAsync(hout, dout, out_bytes, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(bootstrap results)");
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "bootstrap_kernel");
  memcpy(job->medians, hout, G * M * 8);
  memcpy(job->ci_lo, hout + align256(G * M * 8), G * M * 8);
  memcpy(job->ci_hi, hout + 2 * align256(G * M * 8), G * M * 8);
  return PM_OK;
}

int pm_analyze_sweep(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out, pm_bootstrap_job* groups) {
  if (!trials || !policy || !out || !groups) return fail(PM_E_INVALID, "NULL argument");
  if (policy->min_samples < 2) return fail(PM_E_INVALID, "min_samples must be >= 2");
  if (trials->n_trials < 0) return fail(PM_E_INVALID, "negative n_trials");
  pm_bootstrap_job J = *groups;
  J.n_rows = trials->n_trials; J.n_metrics = PM_N_METRICS;
  const size_t G = J.n_groups < 0 ? 0 : (size_t)J.n_groups, M = PM_N_METRICS, n = (size_t)trials->n_trials;
  if (J.n_groups < 0 || J.n_members < 0) return fail(PM_E_INVALID, "negative group sizes");
  if (J.resamples < 40 || J.resamples > (1 << 24)) return fail(PM_E_INVALID, "resamples must be in [40, 2^24]");
  if (!J.group_offsets || !J.seeds || !J.medians || !J.ci_lo || !J.ci_hi) return fail(PM_E_INVALID, "a group array is NULL");
  int mm = 0;
  for (size_t g = 0; g < G; ++g) {
    const int c = J.group_offsets[g + 1] - J.group_offsets[g];
    if (c < 0) return fail(PM_E_INVALID, "group_offsets must be non-decreasing");
    if (c > kMaxGroupMembers) return fail(PM_E_LIMIT, "group %zu lists %d members; the limit is %d", g, c, kMaxGroupMembers);
    if (c > mm) mm = c;
  }
  if (G && (J.group_offsets[0] != 0 || J.group_offsets[G] != J.n_members))
    return fail(PM_E_INVALID, "group_offsets must start at 0 and end at n_members");
  for (int i = 0; i < J.n_members; ++i)
    if (J.member_rows && (J.member_rows[i] < 0 || (size_t)J.member_rows[i] >= n)) return fail(PM_E_INVALID, "member_rows[%d] out of range", i);
  int device = 0, rc = current_device(&device);
  if (rc) return rc;
  if (prepare_bootstrap_constants(device)) return fail(PM_E_CUDA, "bootstrap constants upload failed");
  if (n == 0) return PM_OK;
  if (G && (rc = check_bootstrap_fits((int)M, mm))) return rc;
  const size_t gin = align256((G + 1) * 4) + align256((size_t)J.n_members * 4) + align256(G * 8);
  const size_t gout = 3 * align256(G * M * 8);
  const size_t bscratch = bootstrap_scratch_bytes((int)G, mm, J.resamples);
  Arena& A = g_arenas[device];
  std::lock_guard<std::mutex> guard(A.lock);
  StagedTrials S;
  if ((rc = plan_trials(*trials, S))) return rc;
  // extra host bytes hold the group inputs then outputs; extra device bytes mirror them plus scratch
  if ((rc = arena_reserve(A, S.end + S.scratch + gin + gout + bscratch, S.end + gin + gout))) return rc;
  place_results(A, n, gin + gout + bscratch, S);
  char* hbase = static_cast<char*>(A.host) + S.end;
  char* dbase = static_cast<char*>(A.dev) + S.end;
  Layout hl{hbase};
  int32_t* ho; int32_t* hr; uint64_t* hs;
  hl.place(ho, G + 1); memcpy(ho, J.group_offsets, (G + 1) * 4);
  hl.place(hr, J.n_members); if (J.member_rows) memcpy(hr, J.member_rows, (size_t)J.n_members * 4);
  else for (int i = 0; i < J.n_members; ++i) hr[i] = i;
  hl.place(hs, G); memcpy(hs, J.seeds, G * 8);
  auto dptr = [&](const void* h) { return dbase + (static_cast<const char*>(h) - hbase); };
  char* dout = dbase + gin;
  BootArgs args{(int)G, (int)M, J.resamples, mm, S.dres.metrics, reinterpret_cast<const int32_t*>(dptr(ho)),
                reinterpret_cast<const int32_t*>(dptr(hr)), S.dres.valid, reinterpret_cast<const uint64_t*>(dptr(hs)),
                reinterpret_cast<double*>(dout), reinterpret_cast<double*>(dout + align256(G * M * 8)),
                reinterpret_cast<double*>(dout + 2 * align256(G * M * 8)),
                reinterpret_cast<uint8_t*>(dout + gout), 1, 1};
  // The resample draws need only seeds and group sizes: their inputs go first,
  // on the side stream, and the draws run there while the host stages the
  // trials (the GPU is otherwise idle then); the fold waits for them.
  cudaError_t e = cudaSuccess;
  if (G) {
    e = cudaMemcpyAsync(dbase, hbase, gin, cudaMemcpyHostToDevice, A.side);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(groups)");
    launch_bootstrap_prepare(args, A.side);
    e = cudaEventRecord(A.join, A.side);
    if (e != cudaSuccess) { cudaStreamSynchronize(A.side); return cuda_fail(e, "join record"); }
  }
  if ((rc = copy_trials(A, *trials, S))) {
    cudaStreamSynchronize(A.side);   // the draws use the arena: done before it is reused
    return rc;
  }
  launch_analyze(S.dev, *policy, S.dres, S.max_cov, S.gscratch, A.stream, nullptr);
  // Per-trial results leave on the side stream while the fold runs; the host
  // copies them out while the fold's results are still on their way.
  e = cudaEventRecord(A.analysed, A.stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(A.side, A.analysed, 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(static_cast<char*>(A.host) + S.in_bytes, static_cast<char*>(A.dev) + S.in_bytes, S.res_bytes,
                        cudaMemcpyDeviceToHost, A.side);
  if (e == cudaSuccess) e = cudaEventRecord(A.results, A.side);
  if (e == cudaSuccess && G) e = cudaStreamWaitEvent(A.stream, A.join, 0);
  if (e == cudaSuccess && G) {
    launch_bootstrap(args, A.stream);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(hbase + gin, dout, gout, cudaMemcpyDeviceToHost, A.stream);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaStreamSynchronize(A.side);
    cudaStreamSynchronize(A.stream);
    return cuda_fail(e, "sweep kernels and copies");
  }
  e = cudaEventSynchronize(A.results);
  if (e == cudaSuccess) copy_results_out(S, n, out);
  const cudaError_t e2 = cudaStreamSynchronize(A.stream);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    cudaStreamSynchronize(A.side);
    return cuda_fail(e != cudaSuccess ? e : e2, "sweep kernels");
  }
  if (G) {
    memcpy(groups->medians, hbase + gin, G * M * 8);
    memcpy(groups->ci_lo, hbase + gin + align256(G * M * 8), G * M * 8);
    memcpy(groups->ci_hi, hbase + gin + 2 * align256(G * M * 8), G * M * 8);
  }
  groups->n_rows = (int32_t)n; groups->n_metrics = PM_N_METRICS; groups->max_members = mm;
  return PM_OK;
}

int pm_resample_indices(uint64_t seed, int32_t n, int32_t resamples, int32_t* out) {
  if (!out || n < 1 || n > kMaxGroupMembers || resamples < 1 || (int64_t)n * resamples > (1 << 26))
    return fail(PM_E_INVALID, "pm_resample_indices: n in [1, %d], resamples >= 1, n*resamples <= 2^26", kMaxGroupMembers);
  int device = 0, rc = current_device(&device);
  if (rc) return rc;
  if (prepare_bootstrap_constants(device)) return fail(PM_E_CUDA, "bootstrap constants upload failed");
  const size_t bytes = (size_t)n * resamples * 4;
  Arena& A = g_arenas[device];
  std::lock_guard<std::mutex> guard(A.lock);
  if ((rc = arena_reserve(A, bytes, bytes))) return rc;
  launch_resample_indices(seed, n, resamples, static_cast<int32_t*>(A.dev), A.stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "resample_indices launch");
  e = cudaMemcpyAsync(A.host, A.dev, bytes, cudaMemcpyDeviceToHost, A.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(A.stream);
  if (e != cudaSuccess) return cuda_fail(e, "resample_indices");
  memcpy(out, A.host, bytes);
  return PM_OK;
}

}  // extern "C"
