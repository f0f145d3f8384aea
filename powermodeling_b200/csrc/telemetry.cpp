// NVML telemetry: device handles, one-sample reads and the sampling thread.
//
// Restates powermodeling/telemetry.py (NvmlDevice.read_sample 195-243, its
// field handling 119-193, Sampler 341-438) as native code: the sample is read
// into a fixed struct (pmb200_telemetry.h) with the per-field error codes the
// Python dictionary carries, and the sampler is a std::thread with the same
// tick rule (a fixed deadline advanced by the interval; missed ticks are
// skipped, not caught up), the same first-sample handshake, the same final
// bracket sample on stop and the same stop on a fatal NVML code.  The default
// backend is libnvidia-ml.so.1, opened with dlopen so the library loads on a
// machine without a driver.
#include <dlfcn.h>
#include <strings.h>
#include <time.h>

#include <nvml.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "pmb200.h"
#include "pmb200_telemetry.h"

namespace pm {
int fail(int code, const char* fmt, ...);
}
using pm::fail;

namespace {

double monotonic_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return double(ts.tv_sec) + double(ts.tv_nsec) * 1e-9;
}

double realtime_s() {
  timespec ts;
  clock_gettime(CLOCK_REALTIME, &ts);
  return double(ts.tv_sec) + double(ts.tv_nsec) * 1e-9;
}

// ---------------------------------------------------------------- libnvidia-ml backend
struct NvmlApi {
  void* so = nullptr;
  bool loaded = false;
  std::string error;
  decltype(&nvmlInit_v2) init = nullptr;
  decltype(&nvmlShutdown) shutdown = nullptr;
  decltype(&nvmlErrorString) error_string = nullptr;
  decltype(&nvmlDeviceGetHandleByUUID) by_uuid = nullptr;
  decltype(&nvmlDeviceGetHandleByIndex_v2) by_index = nullptr;
  decltype(&nvmlDeviceGetUUID) uuid = nullptr;
  decltype(&nvmlDeviceGetPowerUsage) power_usage = nullptr;
  decltype(&nvmlDeviceGetFieldValues) field_values = nullptr;
  decltype(&nvmlDeviceGetTotalEnergyConsumption) energy = nullptr;
  decltype(&nvmlDeviceGetClockInfo) clock = nullptr;
  decltype(&nvmlDeviceGetTemperature) temperature = nullptr;
  decltype(&nvmlDeviceGetPerformanceState) pstate = nullptr;
  decltype(&nvmlDeviceGetCurrentClocksEventReasons) event_reasons = nullptr;
  decltype(&nvmlDeviceGetCurrentClocksThrottleReasons) throttle_reasons = nullptr;
  decltype(&nvmlDeviceGetUtilizationRates) utilization = nullptr;
  decltype(&nvmlDeviceGetPowerManagementLimit) power_limit = nullptr;
  decltype(&nvmlDeviceGetEnforcedPowerLimit) enforced_limit = nullptr;
  decltype(&nvmlDeviceGetComputeRunningProcesses_v3) compute_procs = nullptr;
  decltype(&nvmlDeviceGetGraphicsRunningProcesses_v3) graphics_procs = nullptr;
  decltype(&nvmlDeviceGetMPSComputeRunningProcesses_v3) mps_procs = nullptr;
  decltype(&nvmlDeviceGetName) name = nullptr;
  decltype(&nvmlDeviceGetCudaComputeCapability) cc = nullptr;
  decltype(&nvmlDeviceGetMemoryInfo) memory = nullptr;
  decltype(&nvmlDeviceGetPciInfo_v3) pci = nullptr;
  decltype(&nvmlDeviceGetMigMode) mig = nullptr;
  decltype(&nvmlDeviceGetPersistenceMode) persistence = nullptr;
  decltype(&nvmlDeviceGetEccMode) ecc = nullptr;
  decltype(&nvmlDeviceGetPowerManagementLimitConstraints) constraints = nullptr;
  decltype(&nvmlDeviceGetPowerManagementDefaultLimit) default_limit = nullptr;
  decltype(&nvmlSystemGetDriverVersion) driver_version = nullptr;
  decltype(&nvmlSystemGetNVMLVersion) nvml_version = nullptr;
};

std::mutex g_api_lock;
NvmlApi g_api;

template <class F>
void bind(void* so, F& f, const char* name) {
  f = reinterpret_cast<F>(dlsym(so, name));
}

// Loads libnvidia-ml.so.1 once.  Optional entry points stay NULL and read as
// NVML_ERROR_FUNCTION_NOT_FOUND.
NvmlApi* nvml_api() {
  std::lock_guard<std::mutex> guard(g_api_lock);
  if (g_api.loaded) return &g_api;
  if (!g_api.so) {
    g_api.so = dlopen("libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!g_api.so) {
      const char* e = dlerror();
      g_api.error = e ? e : "dlopen(libnvidia-ml.so.1) failed";
      return nullptr;
    }
  }
  void* so = g_api.so;
  bind(so, g_api.init, "nvmlInit_v2");
  bind(so, g_api.shutdown, "nvmlShutdown");
  bind(so, g_api.error_string, "nvmlErrorString");
  bind(so, g_api.by_uuid, "nvmlDeviceGetHandleByUUID");
  bind(so, g_api.by_index, "nvmlDeviceGetHandleByIndex_v2");
  bind(so, g_api.uuid, "nvmlDeviceGetUUID");
  bind(so, g_api.power_usage, "nvmlDeviceGetPowerUsage");
  bind(so, g_api.field_values, "nvmlDeviceGetFieldValues");
  bind(so, g_api.energy, "nvmlDeviceGetTotalEnergyConsumption");
  bind(so, g_api.clock, "nvmlDeviceGetClockInfo");
  bind(so, g_api.temperature, "nvmlDeviceGetTemperature");
  bind(so, g_api.pstate, "nvmlDeviceGetPerformanceState");
  bind(so, g_api.event_reasons, "nvmlDeviceGetCurrentClocksEventReasons");
  bind(so, g_api.throttle_reasons, "nvmlDeviceGetCurrentClocksThrottleReasons");
  bind(so, g_api.utilization, "nvmlDeviceGetUtilizationRates");
  bind(so, g_api.power_limit, "nvmlDeviceGetPowerManagementLimit");
  bind(so, g_api.enforced_limit, "nvmlDeviceGetEnforcedPowerLimit");
  bind(so, g_api.compute_procs, "nvmlDeviceGetComputeRunningProcesses_v3");
  bind(so, g_api.graphics_procs, "nvmlDeviceGetGraphicsRunningProcesses_v3");
  bind(so, g_api.mps_procs, "nvmlDeviceGetMPSComputeRunningProcesses_v3");
  bind(so, g_api.name, "nvmlDeviceGetName");
  bind(so, g_api.cc, "nvmlDeviceGetCudaComputeCapability");
  bind(so, g_api.memory, "nvmlDeviceGetMemoryInfo");
  bind(so, g_api.pci, "nvmlDeviceGetPciInfo_v3");
  bind(so, g_api.mig, "nvmlDeviceGetMigMode");
  bind(so, g_api.persistence, "nvmlDeviceGetPersistenceMode");
  bind(so, g_api.ecc, "nvmlDeviceGetEccMode");
  bind(so, g_api.constraints, "nvmlDeviceGetPowerManagementLimitConstraints");
  bind(so, g_api.default_limit, "nvmlDeviceGetPowerManagementDefaultLimit");
  bind(so, g_api.driver_version, "nvmlSystemGetDriverVersion");
  bind(so, g_api.nvml_version, "nvmlSystemGetNVMLVersion");
  if (!g_api.init || !g_api.shutdown || !g_api.by_index || !g_api.by_uuid || !g_api.uuid) {
    g_api.error = "libnvidia-ml.so.1 lacks nvmlInit_v2/nvmlDeviceGetHandleBy*/nvmlDeviceGetUUID";
    return nullptr;
  }
  g_api.loaded = true;
  return &g_api;
}

constexpr int kNotFound = NVML_ERROR_FUNCTION_NOT_FOUND;
inline nvmlDevice_t H(void* h) { return static_cast<nvmlDevice_t>(h); }

int n_init(void*) { return g_api.init(); }
int n_shutdown(void*) { return g_api.shutdown(); }
int n_by_uuid(void*, const char* uuid, void** h) {
  nvmlDevice_t d{};
  int rc = g_api.by_uuid(uuid, &d);
  *h = d;
  return rc;
}
int n_by_index(void*, uint32_t index, void** h) {
  nvmlDevice_t d{};
  int rc = g_api.by_index(index, &d);
  *h = d;
  return rc;
}
int n_uuid(void*, void* h, char* buf, uint32_t len) { return g_api.uuid(H(h), buf, len); }
int n_power(void*, void* h, double* mw) {
  if (!g_api.power_usage) return kNotFound;
  unsigned v = 0;
  int rc = g_api.power_usage(H(h), &v);
  *mw = v;
  return rc;
}
int n_fields(void*, void* h, int count, pm_nvml_field* f) {
  if (!g_api.field_values) return kNotFound;
  nvmlFieldValue_t v[4];
  if (count > 4) return NVML_ERROR_INVALID_ARGUMENT;
  std::memset(v, 0, sizeof(v));
  for (int i = 0; i < count; ++i) {
    v[i].fieldId = f[i].field_id;
    v[i].scopeId = f[i].scope_id;
  }
  int rc = g_api.field_values(H(h), count, v);
  if (rc) return rc;
  for (int i = 0; i < count; ++i) {
    f[i].field_id = v[i].fieldId;
    f[i].scope_id = v[i].scopeId;
    f[i].timestamp_us = v[i].timestamp;
    f[i].latency_us = v[i].latencyUsec;
    f[i].value_type = int(v[i].valueType);
    f[i].ret = int(v[i].nvmlReturn);
    f[i].value_error = 0;
    f[i].meta_error = 0;
    switch (v[i].valueType) {
      case NVML_VALUE_TYPE_DOUBLE: f[i].value.d = v[i].value.dVal; break;
      case NVML_VALUE_TYPE_UNSIGNED_INT: f[i].value.ui = v[i].value.uiVal; break;
      case NVML_VALUE_TYPE_UNSIGNED_LONG: f[i].value.ul = v[i].value.ulVal; break;
      case NVML_VALUE_TYPE_UNSIGNED_LONG_LONG: f[i].value.ull = v[i].value.ullVal; break;
      case NVML_VALUE_TYPE_SIGNED_LONG_LONG: f[i].value.sll = v[i].value.sllVal; break;
      default: f[i].value.ull = v[i].value.ullVal; break;
    }
  }
  return 0;
}
int n_energy(void*, void* h, uint64_t* mj) {
  if (!g_api.energy) return kNotFound;
  unsigned long long v = 0;
  int rc = g_api.energy(H(h), &v);
  *mj = v;
  return rc;
}
int n_clock(void*, void* h, int kind, uint64_t* mhz) {
  if (!g_api.clock) return kNotFound;
  static const nvmlClockType_t kinds[3] = {NVML_CLOCK_GRAPHICS, NVML_CLOCK_SM, NVML_CLOCK_MEM};
  unsigned v = 0;
  int rc = g_api.clock(H(h), kinds[kind], &v);
  *mhz = v;
  return rc;
}
int n_temperature(void*, void* h, int64_t* c) {
  if (!g_api.temperature) return kNotFound;
  unsigned v = 0;
  int rc = g_api.temperature(H(h), NVML_TEMPERATURE_GPU, &v);
  *c = v;
  return rc;
}
int n_pstate(void*, void* h, int64_t* p) {
  if (!g_api.pstate) return kNotFound;
  nvmlPstates_t v{};
  int rc = g_api.pstate(H(h), &v);
  *p = int64_t(v);
  return rc;
}
int n_throttle(void*, void* h, uint64_t* r) {
  unsigned long long v = 0;
  int rc = g_api.event_reasons ? g_api.event_reasons(H(h), &v)
           : g_api.throttle_reasons ? g_api.throttle_reasons(H(h), &v) : kNotFound;
  *r = v;
  return rc;
}
int n_util(void*, void* h, int64_t* g, int64_t* m) {
  if (!g_api.utilization) return kNotFound;
  nvmlUtilization_t u{};
  int rc = g_api.utilization(H(h), &u);
  *g = u.gpu;
  *m = u.memory;
  return rc;
}
int n_limit(void*, void* h, double* mw) {
  if (!g_api.power_limit) return kNotFound;
  unsigned v = 0;
  int rc = g_api.power_limit(H(h), &v);
  *mw = v;
  return rc;
}
int n_enforced(void*, void* h, double* mw) {
  if (!g_api.enforced_limit) return kNotFound;
  unsigned v = 0;
  int rc = g_api.enforced_limit(H(h), &v);
  *mw = v;
  return rc;
}
int n_procs(void*, void* h, int kind, uint32_t* count, pm_nvml_process* out) {
  auto f = kind == 0 ? g_api.compute_procs : kind == 1 ? g_api.graphics_procs : g_api.mps_procs;
  if (!f) return kNotFound;
  std::vector<nvmlProcessInfo_t> info(*count ? *count : 1);
  unsigned n = *count;
  int rc = f(H(h), &n, info.data());
  *count = n;
  if (rc) return rc;
  for (unsigned i = 0; i < n; ++i) {
    out[i].pid = info[i].pid;
    out[i].used_bytes = info[i].usedGpuMemory;  // NVML_VALUE_NOT_AVAILABLE is UINT64_MAX
  }
  return 0;
}
int n_fatal(void*, int code) {
  return code == NVML_ERROR_UNINITIALIZED || code == NVML_ERROR_GPU_IS_LOST || code == NVML_ERROR_RESET_REQUIRED ||
         code == NVML_ERROR_LIB_RM_VERSION_MISMATCH;
}

pm_nvml_backend native_backend() {
  pm_nvml_backend b{};
  b.ctx = &g_api;
  b.init = n_init;
  b.shutdown = n_shutdown;
  b.handle_by_uuid = n_by_uuid;
  b.handle_by_index = n_by_index;
  b.uuid = n_uuid;
  b.power_usage = n_power;
  b.field_values = n_fields;
  b.total_energy = n_energy;
  b.clock = n_clock;
  b.temperature = n_temperature;
  b.pstate = n_pstate;
  b.throttle_reasons = n_throttle;
  b.utilization = n_util;
  b.power_limit = n_limit;
  b.enforced_power_limit = n_enforced;
  b.processes = n_procs;
  b.is_fatal = n_fatal;
  const uint32_t ids[4] = {NVML_FI_DEV_POWER_INSTANT, NVML_FI_DEV_POWER_AVERAGE, NVML_FI_DEV_POWER_INSTANT,
                           NVML_FI_DEV_POWER_AVERAGE};
  const uint32_t scopes[4] = {NVML_POWER_SCOPE_GPU, NVML_POWER_SCOPE_GPU, NVML_POWER_SCOPE_MEMORY,
                              NVML_POWER_SCOPE_MEMORY};
  for (int i = 0; i < 4; ++i) {
    b.field_id[i] = ids[i];
    b.scope_id[i] = scopes[i];
    b.field_missing[i] = 0;
  }
  return b;
}

// Init/shutdown reference counts per backend context: one nvmlInit for all
// devices opened through the same backend, nvmlShutdown when the last closes.
std::mutex g_session_lock;
std::map<void*, int> g_sessions;

}  // namespace

struct pm_nvml_device {
  pm_nvml_backend be{};
  bool native = false;
  void* handle = nullptr;
  char uuid[96] = {};
  std::timed_mutex lock;
  bool closed = false;
  std::atomic<int> active_samplers{0};
  bool have_energy = false;
  uint64_t last_energy = 0;
};

namespace {

constexpr auto kLockWait = std::chrono::seconds(1);

void release_session(const pm_nvml_backend& be) {
  std::lock_guard<std::mutex> guard(g_session_lock);
  auto it = g_sessions.find(be.ctx);
  if (it == g_sessions.end()) return;
  if (it->second <= 1) {
    g_sessions.erase(it);
    be.shutdown(be.ctx);
  } else {
    --it->second;
  }
}

bool finite_nonneg(double v) { return std::isfinite(v) && v >= 0; }

// Reads one sample with the device lock held.  Field order and checks follow
// telemetry.py:195-243 and, for the power fields, 119-193.
void read_locked(pm_nvml_device* d, pm_nvml_sample* s, std::vector<pm_nvml_process>& procs) {
  const pm_nvml_backend& be = d->be;
  void* ctx = be.ctx;
  void* h = d->handle;
  std::memset(s, 0, sizeof(*s));
  s->query_start_s = monotonic_s();
  s->query_realtime_start_s = realtime_s();

  double mw = 0;
  int rc = be.power_usage(ctx, h, &mw);
  s->power_mw = mw;
  s->code[PM_TF_POWER] = rc ? rc : finite_nonneg(mw) ? 0 : PM_TE_VALUE;

  // Power fields: requested together in one call, checked one by one.
  pm_nvml_field f[4];
  int map[4], pending = 0;
  for (int i = 0; i < 4; ++i) {
    if (be.field_missing[i]) {
      s->code[PM_TF_POWER_INSTANT + i] = be.field_missing[i];
      continue;
    }
    std::memset(&f[pending], 0, sizeof(pm_nvml_field));
    f[pending].field_id = be.field_id[i];
    f[pending].scope_id = be.scope_id[i];
    map[pending++] = i;
  }
  if (pending) {
    s->flags |= PM_TS_FIELDS_QUERIED;
    rc = be.field_values(ctx, h, pending, f);
    if (rc) {
      s->code[PM_TF_FIELD_QUERY] = rc;
      for (int k = 0; k < pending; ++k) s->code[PM_TF_POWER_INSTANT + map[k]] = rc;
    } else {
      for (int k = 0; k < pending; ++k) {
        const int i = map[k];
        const pm_nvml_field& v = f[k];
        int code = 0;
        double value = 0;
        s->field_value_type[i] = v.value_type;
        if (v.ret) {
          code = v.ret;
        } else if (v.field_id != be.field_id[i]) {
          code = PM_TE_FIELD_ID;
        } else if (v.scope_id != be.scope_id[i]) {
          code = PM_TE_FIELD_SCOPE;
        } else if (v.value_type < 0 || v.value_type > 4) {
          code = PM_TE_VALUE_TYPE;
        } else if (v.value_error) {
          code = v.value_error;
        } else {
          switch (v.value_type) {
            case 0: value = v.value.d; break;
            case 1: value = double(v.value.ui); break;
            case 2: value = double(v.value.ul); break;
            case 3: value = double(v.value.ull); break;
            default: value = double(v.value.sll); break;
          }
          if (!finite_nonneg(value)) code = PM_TE_VALUE;
          else if (v.meta_error) code = v.meta_error;
        }
        s->field_mw[i] = value;
        s->field_timestamp_us[i] = v.timestamp_us;
        s->field_latency_us[i] = v.latency_us;
        s->code[PM_TF_POWER_INSTANT + i] = code;
      }
    }
  }

  uint64_t energy = 0;
  rc = be.total_energy(ctx, h, &energy);
  s->energy_mj = energy;
  s->code[PM_TF_ENERGY] = rc;
  if (!rc) {
    if (d->have_energy && energy < d->last_energy) s->flags |= PM_TS_ENERGY_DECREASED;
    d->have_energy = true;
    d->last_energy = energy;
  }
  uint64_t* clocks[3] = {&s->graphics_clock_mhz, &s->sm_clock_mhz, &s->memory_clock_mhz};
  for (int k = 0; k < 3; ++k) s->code[PM_TF_GRAPHICS_CLOCK + k] = be.clock(ctx, h, k, clocks[k]);
  s->code[PM_TF_TEMPERATURE] = be.temperature(ctx, h, &s->temperature_c);
  s->code[PM_TF_PSTATE] = be.pstate(ctx, h, &s->pstate);
  s->code[PM_TF_THROTTLE] = be.throttle_reasons(ctx, h, &s->throttle_reasons);
  s->code[PM_TF_UTILIZATION] =
      be.utilization(ctx, h, &s->gpu_utilization_percent, &s->memory_utilization_percent);
  rc = be.power_limit(ctx, h, &s->power_limit_mw);
  s->code[PM_TF_POWER_LIMIT] = rc ? rc : finite_nonneg(s->power_limit_mw) ? 0 : PM_TE_VALUE;
  rc = be.enforced_power_limit(ctx, h, &s->enforced_power_limit_mw);
  s->code[PM_TF_ENFORCED_LIMIT] = rc ? rc : finite_nonneg(s->enforced_power_limit_mw) ? 0 : PM_TE_VALUE;

  for (int kind = 0; kind < 3; ++kind) {
    const uint32_t base = uint32_t(procs.size());
    uint32_t count = 64;
    procs.resize(base + count);
    rc = be.processes(ctx, h, kind, &count, procs.data() + base);
    if (rc == NVML_ERROR_INSUFFICIENT_SIZE && count > 64 && count < (1u << 20)) {
      procs.resize(base + count);
      rc = be.processes(ctx, h, kind, &count, procs.data() + base);
    }
    if (rc) count = 0;
    for (uint32_t i = 0; i < count && !rc; ++i)
      if (procs[base + i].pid == 0) rc = PM_TE_PID;
    if (rc) count = 0;
    procs.resize(base + count);
    s->process_offset[kind] = base;
    s->process_count[kind] = count;
    s->code[PM_TF_COMPUTE_PROCS + kind] = rc;
  }

  s->query_end_s = monotonic_s();
  s->query_realtime_end_s = realtime_s();
  s->t_s = (s->query_start_s + s->query_end_s) / 2;
  s->query_duration_s = s->query_end_s - s->query_start_s;
  for (int k = 0; k < PM_TF_COUNT; ++k) {
    const int c = s->code[k];
    if (c && !(c >= 0x10000 && c < PM_TE_FOREIGN_BASE) && be.is_fatal(ctx, c)) s->flags |= PM_TS_FATAL;
  }
}

// 0, or PM_TE_LOCK / PM_TE_CLOSED when no read took place.
int read_sample(pm_nvml_device* d, pm_nvml_sample* s, std::vector<pm_nvml_process>& procs) {
  std::unique_lock<std::timed_mutex> guard(d->lock, std::defer_lock);
  if (!guard.try_lock_for(kLockWait)) return PM_TE_LOCK;
  if (d->closed) return PM_TE_CLOSED;
  read_locked(d, s, procs);
  return 0;
}

}  // namespace

struct pm_sampler {
  pm_nvml_device* dev = nullptr;
  double interval = 0.02;
  std::thread thread;
  std::mutex m;
  std::condition_variable cv;
  bool launched = false, stop = false, started = false, finished = false, attached = false;
  std::vector<pm_nvml_sample> samples;
  std::vector<pm_nvml_process> procs;
  int reason = 0;
  uint64_t where = 0;

  // Reads and appends one sample; false ends the thread (fatal code or no read).
  bool take() {
    pm_nvml_sample s;
    std::vector<pm_nvml_process> local;
    local.reserve(16);
    const int rc = read_sample(dev, &s, local);
    std::lock_guard<std::mutex> guard(m);
    if (rc) {
      reason = 3;
      where = samples.size();
      return false;
    }
    const uint32_t base = uint32_t(procs.size());
    for (int k = 0; k < 3; ++k) s.process_offset[k] += base;
    procs.insert(procs.end(), local.begin(), local.end());
    s.sequence = uint32_t(samples.size());
    samples.push_back(s);
    if (s.flags & PM_TS_FATAL) {
      reason = 1;
      where = samples.size() - 1;
      return false;
    }
    return true;
  }

  void run() {
    using clock = std::chrono::steady_clock;
    const auto step = std::chrono::duration_cast<clock::duration>(std::chrono::duration<double>(interval));
    bool ok = take();
    if (ok) {
      {
        std::lock_guard<std::mutex> guard(m);
        started = true;
      }
      cv.notify_all();
      auto deadline = clock::now() + step;
      for (;;) {
        {
          std::unique_lock<std::mutex> lk(m);
          if (cv.wait_until(lk, deadline, [&] { return stop; })) break;
        }
        if (!(ok = take())) break;
        const auto now = clock::now();
        deadline += step;  // skip missed ticks instead of spinning after a slow query
        if (deadline <= now) deadline = now + step;
      }
      if (ok) take();  // final bracket sample
    }
    {
      std::lock_guard<std::mutex> guard(m);
      started = true;
      finished = true;
      if (attached) {
        dev->active_samplers.fetch_sub(1);
        attached = false;
      }
    }
    cv.notify_all();
  }
};

namespace {
std::chrono::steady_clock::duration seconds(double s) {
  return std::chrono::duration_cast<std::chrono::steady_clock::duration>(std::chrono::duration<double>(s));
}
}  // namespace

extern "C" {

const char* pm_nvml_error_string(int code) {
  NvmlApi* api = nvml_api();
  if (!api || !api->error_string) return nullptr;
  return api->error_string(nvmlReturn_t(code));
}

int pm_nvml_open(const pm_nvml_backend* backend, uint32_t index, const char* uuid, pm_nvml_device** out) {
  if (!out) return fail(PM_E_INVALID, "pm_nvml_open: NULL output");
  *out = nullptr;
  if (uuid && std::strncmp(uuid, "GPU-", 4) != 0)
    return fail(PM_E_INVALID, "Use a complete physical GPU UUID beginning GPU-; MIG UUIDs are unsupported");
  pm_nvml_backend be;
  bool native = false;
  if (backend) {
    be = *backend;
    if (!be.init || !be.shutdown || !be.handle_by_uuid || !be.handle_by_index || !be.uuid || !be.power_usage ||
        !be.field_values || !be.total_energy || !be.clock || !be.temperature || !be.pstate || !be.throttle_reasons ||
        !be.utilization || !be.power_limit || !be.enforced_power_limit || !be.processes || !be.is_fatal)
      return fail(PM_E_INVALID, "pm_nvml_open: backend table has a NULL entry");
  } else {
    if (!nvml_api()) return fail(PM_E_NVML, "NVML unavailable: %s", g_api.error.c_str());
    be = native_backend();
    native = true;
  }
  {
    std::lock_guard<std::mutex> guard(g_session_lock);
    int& count = g_sessions[be.ctx];
    if (count == 0) {
      const int rc = be.init(be.ctx);
      if (rc) {
        g_sessions.erase(be.ctx);
        return fail(PM_E_NVML, "nvmlInit failed with code %d", rc);
      }
    }
    ++count;
  }
  auto* d = new pm_nvml_device;
  d->be = be;
  d->native = native;
  int rc = uuid ? be.handle_by_uuid(be.ctx, uuid, &d->handle) : be.handle_by_index(be.ctx, index, &d->handle);
  if (!rc) rc = be.uuid(be.ctx, d->handle, d->uuid, sizeof(d->uuid));
  if (rc) {
    release_session(be);
    delete d;
    return fail(PM_E_NVML, "NVML device lookup failed with code %d", rc);
  }
  d->uuid[sizeof(d->uuid) - 1] = 0;
  if (std::strncmp(d->uuid, "GPU-", 4) != 0) {
    release_session(be);
    delete d;
    return fail(PM_E_NVML, "Physical GPU handle required; cannot use a MIG device for board telemetry");
  }
  if (uuid && strcasecmp(uuid, d->uuid) != 0) {
    std::string got = d->uuid;
    release_session(be);
    delete d;
    return fail(PM_E_NVML, "GPU UUID mismatch: requested %s, resolved %s", uuid, got.c_str());
  }
  *out = d;
  return PM_OK;
}

int pm_nvml_close(pm_nvml_device* d) {
  if (!d) return PM_OK;
  if (d->active_samplers.load()) return fail(PM_E_STATE, "Stop all telemetry samplers before closing the device");
  std::unique_lock<std::timed_mutex> guard(d->lock, std::defer_lock);
  if (!guard.try_lock_for(kLockWait)) return fail(PM_E_STATE, "NVML query is still running; device cannot be closed safely");
  if (d->closed) return PM_OK;
  if (d->active_samplers.load()) return fail(PM_E_STATE, "Stop all telemetry samplers before closing the device");
  d->closed = true;
  release_session(d->be);
  return PM_OK;
}

// The device struct itself is freed only with the process: a sampler that
// outlived its stop timeout may still reference it.
int pm_nvml_uuid(const pm_nvml_device* d, char* buf, size_t len) {
  if (!d || !buf || !len) return fail(PM_E_INVALID, "pm_nvml_uuid: bad arguments");
  std::snprintf(buf, len, "%s", d->uuid);
  return PM_OK;
}

int pm_nvml_active_samplers(const pm_nvml_device* d) { return d ? d->active_samplers.load() : 0; }

int pm_nvml_read_sample(pm_nvml_device* d, pm_nvml_sample* out, pm_nvml_process* procs, uint32_t max_procs) {
  if (!d || !out) return fail(PM_E_INVALID, "pm_nvml_read_sample: NULL argument");
  std::vector<pm_nvml_process> list;
  const int rc = read_sample(d, out, list);
  if (rc == PM_TE_LOCK) return fail(PM_E_STATE, "Another NVML query is still running; refusing concurrent driver access");
  if (rc == PM_TE_CLOSED) return fail(PM_E_STATE, "NVML device is closed");
  if (list.size() > max_procs || (!procs && !list.empty()))
    return fail(PM_E_LIMIT, "pm_nvml_read_sample: %zu process entries, room for %u", list.size(), max_procs);
  if (!list.empty()) std::memcpy(procs, list.data(), list.size() * sizeof(pm_nvml_process));
  return PM_OK;
}

int pm_nvml_read_metadata(pm_nvml_device* d, pm_nvml_metadata* m) {
  if (!d || !m) return fail(PM_E_INVALID, "pm_nvml_read_metadata: NULL argument");
  if (!d->native) return fail(PM_E_NVML, "pm_nvml_read_metadata reads libnvidia-ml only");
  std::unique_lock<std::timed_mutex> guard(d->lock, std::defer_lock);
  if (!guard.try_lock_for(kLockWait)) return fail(PM_E_STATE, "Another NVML query is still running; refusing concurrent driver access");
  if (d->closed) return fail(PM_E_STATE, "NVML device is closed");
  std::memset(m, 0, sizeof(*m));
  nvmlDevice_t h = H(d->handle);
  NvmlApi& a = g_api;
  m->code[0] = a.name ? a.name(h, m->name, sizeof(m->name)) : kNotFound;
  int major = 0, minor = 0;
  m->code[1] = a.cc ? a.cc(h, &major, &minor) : kNotFound;
  m->cc_major = major;
  m->cc_minor = minor;
  nvmlMemory_t mem{};
  m->code[2] = a.memory ? a.memory(h, &mem) : kNotFound;
  m->memory_total = mem.total;
  m->memory_used = mem.used;
  m->memory_free = mem.free;
  nvmlPciInfo_t pci{};
  m->code[3] = a.pci ? a.pci(h, &pci) : kNotFound;
  std::snprintf(m->pci_bus_id, sizeof(m->pci_bus_id), "%s", pci.busId);
  unsigned cur = 0, pend = 0;
  m->code[4] = a.mig ? a.mig(h, &cur, &pend) : kNotFound;
  m->mig_current = cur;
  m->mig_pending = pend;
  nvmlEnableState_t pm{};
  m->code[5] = a.persistence ? a.persistence(h, &pm) : kNotFound;
  m->persistence_mode = pm;
  nvmlEnableState_t ec = {}, ep = {};
  m->code[6] = a.ecc ? a.ecc(h, &ec, &ep) : kNotFound;
  m->ecc_current = ec;
  m->ecc_pending = ep;
  unsigned lo = 0, hi = 0;
  m->code[7] = a.constraints ? a.constraints(h, &lo, &hi) : kNotFound;
  m->power_limit_min_mw = lo;
  m->power_limit_max_mw = hi;
  unsigned def = 0;
  m->code[8] = a.default_limit ? a.default_limit(h, &def) : kNotFound;
  m->default_power_limit_mw = def;
  m->code[9] = a.driver_version ? a.driver_version(m->driver_version, sizeof(m->driver_version)) : kNotFound;
  m->code[10] = a.nvml_version ? a.nvml_version(m->nvml_version, sizeof(m->nvml_version)) : kNotFound;
  return PM_OK;
}

int pm_sampler_create(pm_nvml_device* d, double interval_s, pm_sampler** out) {
  if (!d || !out) return fail(PM_E_INVALID, "pm_sampler_create: NULL argument");
  if (!std::isfinite(interval_s) || interval_s < 0.001)
    return fail(PM_E_INVALID, "Telemetry interval must be finite and at least 0.001 seconds");
  auto* s = new pm_sampler;
  s->dev = d;
  s->interval = interval_s;
  s->samples.reserve(1024);
  *out = s;
  return PM_OK;
}

int pm_sampler_start(pm_sampler* s, double timeout_s) {
  if (!s) return fail(PM_E_INVALID, "pm_sampler_start: NULL sampler");
  if (!std::isfinite(timeout_s) || timeout_s <= 0) return fail(PM_E_INVALID, "start timeout must be finite and positive");
  {
    std::lock_guard<std::mutex> guard(s->m);
    if (s->launched) return fail(PM_E_STATE, "Sampler has already been started");
  }
  {
    std::unique_lock<std::timed_mutex> guard(s->dev->lock, std::defer_lock);
    if (!guard.try_lock_for(kLockWait))
      return fail(PM_E_STATE, "Another NVML query is still running; refusing concurrent driver access");
    if (s->dev->closed) return fail(PM_E_STATE, "NVML device is closed");
    s->dev->active_samplers.fetch_add(1);
  }
  {
    std::lock_guard<std::mutex> guard(s->m);
    s->attached = true;
    s->launched = true;
  }
  try {
    s->thread = std::thread([s] { s->run(); });
  } catch (...) {
    std::lock_guard<std::mutex> guard(s->m);
    s->dev->active_samplers.fetch_sub(1);
    s->attached = false;
    s->launched = false;
    return fail(PM_E_STATE, "could not start the sampler thread");
  }
  std::unique_lock<std::mutex> lk(s->m);
  if (!s->cv.wait_for(lk, seconds(timeout_s), [&] { return s->started; })) {
    s->stop = true;
    s->cv.notify_all();
    return fail(PM_E_TIMEOUT, "Initial NVML query did not finish; stop further experiments");
  }
  if (s->reason) return fail(PM_E_NVML, "Initial NVML sample failed");
  return PM_OK;
}

int pm_sampler_stop(pm_sampler* s, double timeout_s) {
  if (!s) return fail(PM_E_INVALID, "pm_sampler_stop: NULL sampler");
  if (!std::isfinite(timeout_s) || timeout_s <= 0)
    return fail(PM_E_INVALID, "Sampler shutdown timeout must be finite and positive");
  {
    std::unique_lock<std::mutex> lk(s->m);
    if (!s->launched) return fail(PM_E_STATE, "Sampler has not been started");
    s->stop = true;
    s->cv.notify_all();
    if (!s->cv.wait_for(lk, seconds(timeout_s), [&] { return s->finished; }))
      return fail(PM_E_TIMEOUT, "NVML sampler did not stop; device must remain open until its query finishes");
  }
  if (s->thread.joinable()) s->thread.join();
  std::lock_guard<std::mutex> guard(s->m);
  if (s->reason) return fail(PM_E_NVML, "NVML sampler failed");
  return PM_OK;
}

int pm_sampler_count(pm_sampler* s, uint64_t* samples, uint64_t* processes) {
  if (!s) return fail(PM_E_INVALID, "pm_sampler_count: NULL sampler");
  std::lock_guard<std::mutex> guard(s->m);
  if (samples) *samples = s->samples.size();
  if (processes) *processes = s->procs.size();
  return PM_OK;
}

int pm_sampler_copy(pm_sampler* s, uint64_t first, uint64_t count, pm_nvml_sample* out, pm_nvml_process* procs,
                    uint64_t max_procs) {
  if (!s || (count && !out)) return fail(PM_E_INVALID, "pm_sampler_copy: NULL argument");
  std::lock_guard<std::mutex> guard(s->m);
  if (first > s->samples.size() || count > s->samples.size() - first)
    return fail(PM_E_INVALID, "pm_sampler_copy: samples [%llu, %llu) beyond %zu", (unsigned long long)first,
                (unsigned long long)(first + count), s->samples.size());
  if (count) std::memcpy(out, s->samples.data() + first, count * sizeof(pm_nvml_sample));
  if (procs) {
    const uint64_t n = std::min<uint64_t>(max_procs, s->procs.size());
    if (n) std::memcpy(procs, s->procs.data(), n * sizeof(pm_nvml_process));
  }
  return PM_OK;
}

int pm_sampler_status(pm_sampler* s, int* reason, uint64_t* where, int* running) {
  if (!s) return fail(PM_E_INVALID, "pm_sampler_status: NULL sampler");
  std::lock_guard<std::mutex> guard(s->m);
  if (reason) *reason = s->reason;
  if (where) *where = s->where;
  if (running) *running = s->launched && !s->finished;
  return PM_OK;
}

// A light clock watch: a native thread reads only the SM clock and the clock-event reasons
// (two driver calls of a few microseconds, no energy counter or process lists), so that a timed
// region of a few milliseconds still gets many clock records.
struct pm_clock_watch {
  pm_nvml_device* dev = nullptr;
  std::thread thread;
  std::atomic<bool> stop{false};
  std::chrono::nanoseconds interval{100000};
  std::vector<uint32_t> mhz;
  std::vector<uint64_t> reasons;
  std::vector<double> t;
  std::vector<int> code;
};

int pm_clock_watch_start(pm_nvml_device* d, double interval_s, pm_clock_watch** out) {
  if (!d || !out || !(interval_s > 0) || interval_s > 10) return fail(PM_E_INVALID, "pm_clock_watch_start: bad argument");
  auto* w = new pm_clock_watch();
  w->dev = d;
  w->interval = std::chrono::nanoseconds(int64_t(interval_s * 1e9));
  w->mhz.reserve(1 << 16);
  w->reasons.reserve(1 << 16);
  w->t.reserve(1 << 16);
  w->code.reserve(1 << 16);
  d->active_samplers.fetch_add(1);
  w->thread = std::thread([w] {
    const pm_nvml_backend& be = w->dev->be;
    auto next = std::chrono::steady_clock::now();
    while (!w->stop.load(std::memory_order_relaxed) && w->t.size() < (size_t(1) << 20)) {
      uint64_t mhz = 0, bits = 0;
      int rc = 0;
      {
        std::unique_lock<std::timed_mutex> guard(w->dev->lock, std::defer_lock);
        if (!guard.try_lock_for(kLockWait)) break;
        rc = be.clock(be.ctx, w->dev->handle, 1, &mhz);
        if (!rc) rc = be.throttle_reasons(be.ctx, w->dev->handle, &bits);
      }
      timespec ts;
      clock_gettime(CLOCK_MONOTONIC, &ts);
      w->mhz.push_back(uint32_t(mhz));
      w->reasons.push_back(bits);
      w->t.push_back(double(ts.tv_sec) + ts.tv_nsec * 1e-9);
      w->code.push_back(rc);
      next += w->interval;
      std::this_thread::sleep_until(next);
    }
  });
  *out = w;
  return PM_OK;
}

int pm_clock_watch_stop(pm_clock_watch* w, uint32_t* sm_mhz, uint64_t* reasons, double* t_s, int32_t* codes,
                        uint64_t capacity, uint64_t* count) {
  if (!w || !count) return fail(PM_E_INVALID, "pm_clock_watch_stop: bad argument");
  w->stop.store(true);
  if (w->thread.joinable()) w->thread.join();
  w->dev->active_samplers.fetch_sub(1);
  const uint64_t n = std::min<uint64_t>(w->t.size(), capacity);
  for (uint64_t k = 0; k < n; ++k) {
    if (sm_mhz) sm_mhz[k] = w->mhz[k];
    if (reasons) reasons[k] = w->reasons[k];
    if (t_s) t_s[k] = w->t[k];
    if (codes) codes[k] = w->code[k];
  }
  *count = n;
  delete w;
  return PM_OK;
}

int pm_sampler_destroy(pm_sampler* s) {
  if (!s) return PM_OK;
  {
    std::lock_guard<std::mutex> guard(s->m);
    if (s->launched && !s->finished) return fail(PM_E_STATE, "sampler thread still running; stop it first");
  }
  if (s->thread.joinable()) s->thread.join();
  delete s;
  return PM_OK;
}

}  // extern "C"
