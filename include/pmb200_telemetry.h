/* NVML telemetry sampler: C ABI of libpmb200.so.
 *
 * Replaces the Python telemetry of powermodeling (powermodeling/telemetry.py):
 *   pm_nvml_open / pm_nvml_close      NvmlDevice.__init__ / close        telemetry.py:58-89, 309-330
 *   pm_nvml_read_sample               NvmlDevice.read_sample             telemetry.py:195-243
 *   pm_nvml_read_metadata             NvmlDevice.metadata (raw reads)    telemetry.py:274-308
 *   pm_sampler_*                      Sampler (thread + bracket samples) telemetry.py:341-438
 *
 * The sampler is a native thread that reads the sample fields every tick,
 * timestamps each query with CLOCK_MONOTONIC (midpoint, start, end) and
 * CLOCK_REALTIME (start, end), skips missed ticks, takes a final bracket
 * sample on stop, and stops on a fatal NVML code.  NVML is reached through a
 * backend table: NULL selects libnvidia-ml.so.1 (dlopen at pm_nvml_open), a
 * caller-provided table stands in for the driver (the counterpart of the
 * reference's nvml_module injection hook).
 *
 * Status convention as in pmb200.h: 0 on success, a negative PM_E_* code on
 * failure, message via pm_last_error.  Per-field read errors are not call
 * failures: they are reported in the sample's code[] slots.
 */
#ifndef PMB200_TELEMETRY_H
#define PMB200_TELEMETRY_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-field codes in pm_nvml_sample.code[]: 0 = read, 1..0xFFFF = the NVML
 * return code of the failing call, PM_TE_* = a check of this library failed,
 * >= PM_TE_FOREIGN_BASE = an error the backend table recorded itself (the
 * backend maps the code back to its own description). */
enum {
  PM_TE_OK = 0,
  PM_TE_VALUE = 0x10001,        /* value negative or not finite */
  PM_TE_FIELD_COUNT = 0x10002,  /* field query returned the wrong number of values */
  PM_TE_FIELD_ID = 0x10003,     /* field returned with the wrong field ID */
  PM_TE_FIELD_SCOPE = 0x10004,  /* field returned with the wrong power scope */
  PM_TE_VALUE_TYPE = 0x10005,   /* unsupported NVML value type */
  PM_TE_LOCK = 0x10006,         /* another query held the device for 1 s */
  PM_TE_PID = 0x10007,          /* process inventory holds process ID 0 */
  PM_TE_CLOSED = 0x10008,       /* the device was closed */
  PM_TE_FOREIGN_BASE = 0x1000000
};

/* Sample fields, in the order of the reference's sample dictionary. */
enum {
  PM_TF_POWER = 0,              /* power_w                 nvmlDeviceGetPowerUsage */
  PM_TF_POWER_INSTANT,          /* power_instant_w         field 186, GPU scope */
  PM_TF_POWER_AVERAGE,          /* power_average_w         field 185, GPU scope */
  PM_TF_MEMORY_INSTANT,         /* memory_power_instant_w  field 186, memory scope */
  PM_TF_MEMORY_AVERAGE,         /* memory_power_average_w  field 185, memory scope */
  PM_TF_ENERGY,                 /* energy_mj               nvmlDeviceGetTotalEnergyConsumption */
  PM_TF_GRAPHICS_CLOCK,         /* graphics_clock_mhz */
  PM_TF_SM_CLOCK,               /* sm_clock_mhz */
  PM_TF_MEMORY_CLOCK,           /* memory_clock_mhz */
  PM_TF_TEMPERATURE,            /* temperature_c */
  PM_TF_PSTATE,                 /* pstate */
  PM_TF_THROTTLE,               /* throttle_reasons (clocks event reasons) */
  PM_TF_UTILIZATION,            /* utilization */
  PM_TF_POWER_LIMIT,            /* power_limit_w */
  PM_TF_ENFORCED_LIMIT,         /* enforced_power_limit_w */
  PM_TF_COMPUTE_PROCS,          /* compute_processes */
  PM_TF_GRAPHICS_PROCS,         /* graphics_processes */
  PM_TF_MPS_PROCS,              /* mps_compute_processes */
  PM_TF_FIELD_QUERY,            /* the one nvmlDeviceGetFieldValues call (whole-call failure) */
  PM_TF_COUNT
};

/* pm_nvml_sample.flags */
enum {
  PM_TS_ENERGY_DECREASED = 1u << 0,  /* energy counter went backwards since the previous read */
  PM_TS_FATAL = 1u << 1,             /* a field failed with a fatal NVML code */
  PM_TS_FIELDS_QUERIED = 1u << 2     /* at least one power field was requested */
};

/* One field value as NVML's nvmlFieldValue_t carries it. */
typedef struct pm_nvml_field {
  uint32_t field_id;    /* in: requested; out: as returned */
  uint32_t scope_id;    /* in: requested; out: as returned */
  int64_t timestamp_us; /* unix epoch microseconds */
  int64_t latency_us;
  int32_t value_type;   /* 0 double, 1 uint, 2 ulong, 3 ull, 4 sll */
  int32_t ret;          /* NVML return code of this field */
  int32_t value_error;  /* 0, or a foreign code: the value has no representation of value_type */
  int32_t meta_error;   /* 0, or a foreign code: timestamp/latency not representable */
  union { double d; uint32_t ui; uint64_t ul; uint64_t ull; int64_t sll; } value;
} pm_nvml_field;

typedef struct pm_nvml_process {
  uint64_t pid;
  uint64_t used_bytes;  /* UINT64_MAX = not available */
} pm_nvml_process;

/* Backend table.  Every call returns 0 or an error code (NVML code, or a
 * foreign code >= PM_TE_FOREIGN_BASE).  clock kinds: 0 graphics, 1 SM,
 * 2 memory; process kinds: 0 compute, 1 graphics, 2 MPS.  For process lists
 * *count holds the capacity on entry and the number of entries on return. */
typedef struct pm_nvml_backend {
  void* ctx;
  int (*init)(void* ctx);
  int (*shutdown)(void* ctx);
  int (*handle_by_uuid)(void* ctx, const char* uuid, void** handle);
  int (*handle_by_index)(void* ctx, uint32_t index, void** handle);
  int (*uuid)(void* ctx, void* handle, char* buf, uint32_t len);
  int (*power_usage)(void* ctx, void* handle, double* milliwatts);
  int (*field_values)(void* ctx, void* handle, int count, pm_nvml_field* fields);
  int (*total_energy)(void* ctx, void* handle, uint64_t* millijoules);
  int (*clock)(void* ctx, void* handle, int kind, uint64_t* mhz);
  int (*temperature)(void* ctx, void* handle, int64_t* celsius);
  int (*pstate)(void* ctx, void* handle, int64_t* pstate);
  int (*throttle_reasons)(void* ctx, void* handle, uint64_t* reasons);
  int (*utilization)(void* ctx, void* handle, int64_t* gpu_percent, int64_t* memory_percent);
  int (*power_limit)(void* ctx, void* handle, double* milliwatts);
  int (*enforced_power_limit)(void* ctx, void* handle, double* milliwatts);
  int (*processes)(void* ctx, void* handle, int kind, uint32_t* count, pm_nvml_process* out);
  /* 1 if the code ends the sampler (GPU lost, reset required, ...). */
  int (*is_fatal)(void* ctx, int code);
  /* Field IDs and power scopes for instant GPU, average GPU, instant memory,
   * average memory; a nonzero field_missing[i] (a foreign code) drops that
   * field from the query with that error. */
  uint32_t field_id[4];
  uint32_t scope_id[4];
  int32_t field_missing[4];
} pm_nvml_backend;

/* One sample.  Values whose code[] slot is nonzero are undefined. */
typedef struct pm_nvml_sample {
  double t_s, query_start_s, query_end_s, query_duration_s;  /* CLOCK_MONOTONIC seconds */
  double query_realtime_start_s, query_realtime_end_s;       /* CLOCK_REALTIME seconds */
  double power_mw;                 /* PM_TF_POWER */
  double field_mw[4];              /* PM_TF_POWER_INSTANT .. PM_TF_MEMORY_AVERAGE (raw, milliwatts) */
  int64_t field_timestamp_us[4];
  int64_t field_latency_us[4];
  uint64_t energy_mj;
  uint64_t graphics_clock_mhz, sm_clock_mhz, memory_clock_mhz;
  int64_t temperature_c, pstate;
  uint64_t throttle_reasons;
  int64_t gpu_utilization_percent, memory_utilization_percent;
  double power_limit_mw, enforced_power_limit_mw;
  uint32_t process_offset[3];      /* into the process table of the sampler (or the read buffer) */
  uint32_t process_count[3];
  int32_t code[PM_TF_COUNT];
  int32_t field_value_type[4];     /* value type of each power field as returned */
  uint32_t flags;                  /* PM_TS_* */
  uint32_t sequence;               /* index of the sample in its sampler (0 for single reads) */
} pm_nvml_sample;

typedef struct pm_nvml_metadata {
  char name[96];
  char pci_bus_id[32];
  char driver_version[80];
  char nvml_version[80];
  int64_t cc_major, cc_minor;
  uint64_t memory_total, memory_used, memory_free;
  int64_t mig_current, mig_pending;
  int64_t persistence_mode;
  int64_t ecc_current, ecc_pending;
  double power_limit_min_mw, power_limit_max_mw;
  double default_power_limit_mw;
  /* 0 or error code per item: name, cc, memory, pci, mig, persistence, ecc,
   * constraints, default limit, driver version, nvml version. */
  int32_t code[11];
} pm_nvml_metadata;

typedef struct pm_nvml_device pm_nvml_device;
typedef struct pm_sampler pm_sampler;

/* Opens a device by exact UUID (uuid != NULL, must start with "GPU-") or by
 * NVML index.  backend == NULL: libnvidia-ml.so.1.  The backend's init is
 * called once per backend context across open devices; shutdown when the last
 * one closes. */
int pm_nvml_open(const pm_nvml_backend* backend, uint32_t index, const char* uuid, pm_nvml_device** out);
/* Fails while a sampler is attached, or when a query holds the device for 1 s. */
int pm_nvml_close(pm_nvml_device* device);
int pm_nvml_uuid(const pm_nvml_device* device, char* buf, size_t len);
/* One sample; process entries go to procs[0..max_procs).  Sets
 * PM_TS_ENERGY_DECREASED against the device's previous energy read. */
int pm_nvml_read_sample(pm_nvml_device* device, pm_nvml_sample* out, pm_nvml_process* procs, uint32_t max_procs);
/* Metadata reads (libnvidia-ml backend only; PM_E_NVML with a caller table). */
int pm_nvml_read_metadata(pm_nvml_device* device, pm_nvml_metadata* out);
/* Number of samplers attached to the device. */
int pm_nvml_active_samplers(const pm_nvml_device* device);
/* Text of an NVML return code from the libnvidia-ml backend (NULL otherwise). */
const char* pm_nvml_error_string(int code);

/* interval_s >= 0.001. */
int pm_sampler_create(pm_nvml_device* device, double interval_s, pm_sampler** out);
/* Starts the thread and waits up to timeout_s for the first sample. */
int pm_sampler_start(pm_sampler* sampler, double timeout_s);
/* Signals the thread and waits up to timeout_s for it (final bracket sample
 * included).  PM_E_TIMEOUT when it is still in a query: the sampler stays
 * attached and stop may be called again. */
int pm_sampler_stop(pm_sampler* sampler, double timeout_s);
/* Samples and process entries recorded so far. */
int pm_sampler_count(pm_sampler* sampler, uint64_t* samples, uint64_t* processes);
int pm_sampler_copy(pm_sampler* sampler, uint64_t first, uint64_t count, pm_nvml_sample* out,
                    pm_nvml_process* procs, uint64_t max_procs);
/* Why the thread ended: 0 none, 1 fatal field code (sample index in *where),
 * 2 the start wait timed out, 3 a device query could not take the lock. */
int pm_sampler_status(pm_sampler* sampler, int* reason, uint64_t* where, int* running);
/* Frees the sampler; PM_E_STATE while its thread runs. */
int pm_sampler_destroy(pm_sampler* sampler);

/* A clock watch: a native thread that reads only the SM clock (MHz) and the
 * clock-event reason bits every interval_s (the reference samples them inside
 * its full reads, telemetry.py:195-243; this is the fast form for short timed
 * regions).  The device counts it as an attached sampler until it stops.
 * stop joins the thread, copies up to `capacity` records (any output may be
 * NULL; codes[k] is the driver code of record k, 0 = read) and frees it. */
typedef struct pm_clock_watch pm_clock_watch;
int pm_clock_watch_start(pm_nvml_device* device, double interval_s, pm_clock_watch** out);
int pm_clock_watch_stop(pm_clock_watch* watch, uint32_t* sm_mhz, uint64_t* reasons, double* t_s, int32_t* codes,
                        uint64_t capacity, uint64_t* count);

#ifdef __cplusplus
}
#endif

#endif
