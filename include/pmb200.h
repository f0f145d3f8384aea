/*
 * libpmb200 — B200-native measured-workload and analysis hot path of
 * powermodeling, behind a plain C ABI (no C++ or torch types cross it).
 *
 * Conventions for every entry point:
 *   - return 0 on success, a negative PM_E_* code on failure; the message of
 *     the last failure on the calling thread is copied by pm_last_error();
 *   - no exception crosses the ABI; no entry point keeps a caller pointer;
 *   - "host" entry points take host pointers and copy in and out themselves
 *     (the end-to-end path); "_device" variants take device pointers and a
 *     cudaStream_t passed as void* and never synchronize the stream;
 *   - a floating value that the reference reports as None travels as NaN;
 *     every other floating input is finite (the reference reads a non-finite
 *     number as None).
 *
 * The analysis entry points replace the numeric core of
 * powermodeling/analysis.py (the reference's Python): _interpolate/_integrate
 * (analysis.py:94-124), _phase_stats (127-207), _idle_at (210-216),
 * _measure_epochs (228-276), _paired_reference_contrast (292-423), the
 * numeric body of analyze_trial (597-1056), the group medians of summarize
 * (1455-1470) and _median_ci (1096-1101).  Layout indices (PM_PO_*, PM_TO_*,
 * issue bits) are exported at run time through pm_layout() so bindings never
 * hard-code them.
 */
#ifndef PMB200_H
#define PMB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PM_ABI_VERSION 1

enum {
  PM_OK = 0,
  PM_E_INVALID = -1,     /* bad argument or size */
  PM_E_CUDA = -2,        /* CUDA runtime error */
  PM_E_NODEVICE = -3,    /* no CUDA device visible */
  PM_E_LIMIT = -4,       /* input exceeds a documented maximum */
  PM_E_NVML = -5,        /* NVML unavailable or failed */
  PM_E_TIMEOUT = -6,     /* a bounded device wait gave up */
  PM_E_STATE = -7        /* call out of order for this handle */
};

/* Phase slots of one trial, in the reference's phase names. */
enum { PM_IDLE_PRE = 0, PM_MEASURE = 1, PM_IDLE_POST = 2, PM_REFERENCE = 3, PM_CONTROL = 4, PM_PHASES = 5 };

/* Workload classes (analysis.py:27-31 sets). */
enum { PM_WL_OTHER = 0, PM_WL_TENSOR = 1, PM_WL_MEMORY = 2, PM_WL_SFU = 3, PM_WL_NONLINEAR = 4 };

/* Per-sample flag bits (pm_trials.sample_flags). */
#define PM_S_THROTTLE_VALID   0x0001u /* throttle_reasons parsed to an integer */
#define PM_S_FOREIGN_PID      0x0002u /* inventory pid (not None) differs from the measurement pid */
#define PM_S_NO_COMPUTE_INV   0x0004u /* compute_processes is not a list */
#define PM_S_NO_GRAPHICS_INV  0x0008u /* graphics_processes is not a list */
#define PM_S_MPS              0x0010u /* mps_compute_processes is non-empty */
#define PM_S_PID_UNKNOWN      0x0020u /* an inventory is non-empty while the measurement pid is None */
#define PM_S_ENERGY_ANCHOR    0x0040u /* energy_mj has exact type int (anchor candidate) */
#define PM_S_ENERGY_INT       0x0080u /* energy_mj is a nonnegative integer: use energy_int */
#define PM_S_ENERGY_FLOAT     0x0100u /* energy_mj is a nonnegative float: use energy_float */
#define PM_S_REF_FOREIGN      0x0200u /* some inventory entry's pid (None included) != measurement pid */
#define PM_S_MEMORY_POWER_SET 0x0400u /* memory_power_w is not None */

/* Per-sample columns that may be broadcast (pm_trials.broadcast_columns):
 * a set bit means that array holds one element standing for every sample.
 * t_s is never broadcast. */
enum {
  PM_COL_POWER_W = 1u << 0, PM_COL_MEMORY_POWER_W = 1u << 1, PM_COL_GRAPHICS_CLOCK = 1u << 2,
  PM_COL_SM_CLOCK = 1u << 3, PM_COL_MEMORY_CLOCK = 1u << 4, PM_COL_TEMPERATURE = 1u << 5,
  PM_COL_POWER_LIMIT = 1u << 6, PM_COL_ENFORCED_LIMIT = 1u << 7, PM_COL_PSTATE = 1u << 8,
  PM_COL_ENERGY_INT = 1u << 9, PM_COL_ENERGY_FLOAT = 1u << 10, PM_COL_THROTTLE = 1u << 11,
  PM_COL_SAMPLE_FLAGS = 1u << 12, PM_COL_MEMORY_SOURCE = 1u << 13, PM_COL_ALL = (1u << 14) - 1
};

/* Per-trial flag word (pm_trials.trial_flags). */
#define PM_T_WORKLOAD_MASK       0x0007u /* PM_WL_* */
#define PM_T_HOST_ISSUES         0x0008u /* host-side record checks already failed the trial */
#define PM_T_HOST_BASELINE       0x0010u /* host-side checks found a baseline issue */
#define PM_T_HOST_PAIRED         0x0020u /* host-side protocol/geometry checks found a paired issue */
#define PM_T_ORDER_AB            0x0040u
#define PM_T_ORDER_BA            0x0080u
#define PM_T_TENSOR_PEAK_KNOWN   0x0100u /* trial_scalars[PM_TS_TENSOR_FLOPS_PER_CLOCK] is valid */
#define PM_T_SFU_CONTRACT_OK     0x0200u /* sfu count_issues() returned nothing */
#define PM_T_NONLINEAR_OK        0x0400u /* nonlinear count_issues() returned nothing */
#define PM_T_ROWWISE             0x0800u

/* Epoch list status per (trial, arm), decided while parsing records. */
enum { PM_EP_NONE = 0, PM_EP_OK = 1, PM_EP_INVALID_LIST = 2, PM_EP_NON_DICT_AFTER = 3 };

/* Per-trial scalar slots (pm_trials.trial_scalars, NaN = None). */
enum {
  PM_TS_BENCH_DURATION_S = 0, PM_TS_BENCH_HOST_DURATION_S, PM_TS_BENCH_OPERATIONS, PM_TS_BENCH_LOGICAL_BYTES,
  PM_TS_REF_OPERATIONS, PM_TS_REF_LOGICAL_BYTES,
  PM_TS_REQ_GRAPHICS_MHZ, PM_TS_REQ_MEMORY_MHZ, PM_TS_REQ_SM_MHZ,
  PM_TS_TENSOR_FLOPS_PER_CLOCK, PM_TS_POWER_LIMIT_FALLBACK_W, PM_TS_ROW_WIDTH,
  PM_TS_COUNT
};

typedef struct {
  double trim_s, idle_trim_s, min_measure_s, min_idle_s;
  int32_t min_samples;
  double max_sample_gap_s, clock_tolerance_fraction, max_clock_drift_fraction;
  double max_temperature_drift_c, max_idle_drift_fraction, counter_disagreement_fraction;
} pm_policy;

/*
 * A batch of trials in structure-of-arrays form.  Samples of every
 * (trial, phase) slot are one CSR segment, sorted by strictly increasing t_s
 * (the host applies the reference's last-wins de-duplication, analysis.py:85-91).
 * Every pointer is host memory for pm_analyze_trials and device memory for
 * pm_analyze_trials_device.  A per-sample array holds n_samples elements, or
 * exactly one when its PM_COL_* bit is set in broadcast_columns; the device
 * entry point cannot check device array lengths, so a bit left unset for a
 * one-element array reads past its end.
 */
typedef struct {
  int32_t n_trials;
  int32_t max_phase_samples;       /* longest (trial, phase) segment; the host variant recomputes it */
  int64_t n_samples;
  const int64_t* phase_offsets;    /* [n_trials*PM_PHASES + 1] */
  const double* phase_start_s;     /* [n_trials*PM_PHASES] */
  const double* phase_end_s;
  const uint8_t* phase_present;    /* 1 = phase dict present and non-empty */
  const double* t_s;               /* [n_samples] */
  const double* power_w;
  const double* memory_power_w;
  const double* graphics_clock_mhz;
  const double* sm_clock_mhz;
  const double* memory_clock_mhz;
  const double* temperature_c;
  const double* power_limit_w;
  const double* enforced_power_limit_w;
  const double* pstate;
  const int64_t* energy_int;       /* raw integer counter, two's complement of uint64 */
  const double* energy_float;
  const int64_t* throttle_reasons;
  const uint16_t* sample_flags;
  const uint8_t* memory_power_source; /* 0 = none, 1..15 = host-assigned id of memory_power_source */
  int32_t n_epochs;
  const int32_t* epoch_offsets;    /* [n_trials*2 + 1]; arm 0 measure, arm 1 active_reference */
  const int32_t* epoch_status;     /* [n_trials*2] PM_EP_* */
  const double* epoch_start_s;     /* [n_epochs] */
  const double* epoch_end_s;
  const double* epoch_operations;
  const double* epoch_logical_bytes;
  const double* epoch_loop_slots;
  const uint8_t* epoch_counts_exact;
  const double* trial_scalars;     /* [n_trials*PM_TS_COUNT] */
  const uint32_t* trial_flags;     /* [n_trials] */
  uint32_t broadcast_columns;      /* PM_COL_* bits: those per-sample arrays hold 1 element for all samples */
} pm_trials;

/*
 * Results.  phase_out is [n_trials*PM_PHASES*n_phase_fields] doubles,
 * trial_out [n_trials*n_trial_fields] doubles, issue_bits
 * [n_trials*PM_ISSUE_WORDS] words, metrics [n_trials*n_metrics] in the order
 * of the reference's _METRICS tuple (analysis.py:1059-1074), valid [n_trials].
 * Field counts and slot indices come from pm_layout().
 */
typedef struct {
  double* phase_out;
  uint32_t* phase_flags;           /* [n_trials*PM_PHASES] */
  double* trial_out;
  uint64_t* issue_bits;
  double* metrics;
  uint8_t* valid;
} pm_trial_results;

/* Integer layout constant by name ("PM_PO_COUNT", "PM_TO_BOARD_POWER_W", "PM_I_ACTIVE_THROTTLING", ...);
 * returns -1 for an unknown name. */
int32_t pm_layout(const char* name);

/* Copy of the last error message of the calling thread (truncated to cap). */
size_t pm_last_error(char* buffer, size_t cap);

/* Library and device facts: ABI version, SM count of the current device (0 if none). */
int32_t pm_abi_version(void);
int32_t pm_device_count(void);

/* Analyze a batch of trials: host buffers in, host buffers out (end to end).
 * Staging and device workspaces are owned by the library (grow-only, per device). */
int pm_analyze_trials(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out);
/* Bytes of device scratch pm_analyze_trials_device needs for phases longer
 * than the shared-memory tile (1023 samples); 0 when none is needed.  Device
 * scratch passed to the analysis and bootstrap entry points is 16-byte
 * aligned (the sweep's, pm_analyze_sweep_device, 256-byte aligned). */
size_t pm_analyze_scratch_bytes(int32_t n_trials, int32_t max_phase_samples);
/* Same as pm_analyze_trials with every pointer in device memory, enqueued on
 * `stream`; trials->max_phase_samples must bound every segment. */
int pm_analyze_trials_device(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out,
                             void* scratch, size_t scratch_bytes, void* stream);

/*
 * Group medians and bootstrap confidence intervals (_median_ci,
 * analysis.py:1096-1101, generalised to `resamples` draws with order
 * statistics 25*B/1000-1 and 975*B/1000-1; B=1000 gives the reference's
 * [24] and [974]).
 *   values        [n_rows*n_metrics]: metric rows (NaN = None)
 *   group_offsets [n_groups+1]: group g lists members group_offsets[g]..[g+1]-1
 *                 in the order the reference's bucket holds them
 *   member_rows   [n_members] row of each member in `values` (NULL: member i is row i)
 *   member_valid  [n_rows] rows with 0 are skipped (NULL: all rows count)
 *   seeds         [n_groups]: int(sha256(group_key)[:16], 16), the group's random.Random seed
 *   medians, ci_lo, ci_hi [n_groups*n_metrics] (NaN where the reference gives None)
 * Limits: a group may list at most 128 members; resamples in [40, 2^24].
 */
typedef struct {
  int32_t n_groups, n_metrics, n_members, n_rows, resamples;
  int32_t max_members;             /* largest group; required by the _device variant */
  const double* values;
  const int32_t* group_offsets;
  const int32_t* member_rows;
  const uint8_t* member_valid;
  const uint64_t* seeds;
  double* medians;
  double* ci_lo;
  double* ci_hi;
} pm_bootstrap_job;

int pm_group_bootstrap(const pm_bootstrap_job* job);
/* Device scratch: one prepared multiset histogram per group (6864 bytes)
 * plus every group's index stream (resamples x max_members bytes per group).
 * The _device entry points also accept a scratch without the streams of
 * groups of up to seven members (only the histograms, and the streams when
 * max_members > 7): the prepare pass then consumes the draws as it generates
 * them, which takes several times longer. */
size_t pm_bootstrap_scratch_bytes(int32_t n_groups, int32_t max_members, int32_t resamples);
/* Device buffers, stream-ordered: pm_bootstrap_prepare_device then
 * pm_bootstrap_finish_device, or both at once. */
int pm_group_bootstrap_device(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes, void* stream);
/* The two halves of pm_group_bootstrap_device.  Prepare draws each group's
 * resamples for its listed member count into scratch; it reads only
 * group_offsets and seeds, so it may run on another stream while the metric
 * values are still being computed.  Finish (same job and scratch, ordered
 * after prepare) gathers the values, uses the prepared draws for every metric
 * whose finite count equals the member count, draws afresh for other counts,
 * and writes medians and intervals. */
int pm_bootstrap_prepare_device(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes, void* stream);
int pm_bootstrap_finish_device(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes, void* stream);

/*
 * summarize's numeric core in one call (analysis.py:1400-1470): analyze every
 * trial, then group medians and bootstrap intervals of the _METRICS rows of
 * the trials each group lists, skipping trials the analysis found invalid.
 * Host buffers in and out.  groups->values, ->n_rows, ->n_metrics and
 * ->member_valid are filled by the call (rows are trials, 47 metrics).
 */
int pm_analyze_sweep(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out,
                     pm_bootstrap_job* groups);

/*
 * The same sweep on device buffers, stream-ordered on `stream`: the groups'
 * draws on the library's own side stream (forked from and joined back to
 * `stream`), beside the trial analysis, then the groups' medians and
 * intervals.  The job's values and member_valid are normally out->metrics and
 * out->valid (the groups read the analysis's rows; the finish is ordered after
 * it).  `exchange` (NULL: none; pmb200_peer.h) also stores every group's
 * result into the receiving ranks' gathered tables, as
 * pm_bootstrap_finish_device_exchange does.  One call instead of the
 * analysis, prepare and finish calls: no counterpart in the reference (its
 * summarize is one host call, analysis.py:1400-1470).  Scratch: at least
 * pm_analyze_sweep_scratch_bytes (the analysis's, then the bootstrap's at the
 * next 256-byte boundary).
 */
struct pm_peer_groups;
size_t pm_analyze_sweep_scratch_bytes(int32_t n_trials, int32_t max_phase_samples, int32_t n_groups,
                                      int32_t max_members, int32_t resamples);
int pm_analyze_sweep_device(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out,
                            const pm_bootstrap_job* groups, void* scratch, size_t scratch_bytes,
                            const struct pm_peer_groups* exchange, void* stream);

/*
 * The measured-workload engine behind the powerbench command line
 * (the reference's cuda/gpu_bench.cu main and experiment(), lines 121-254,
 * 519-602, 611-1192, and cuda/sfu.cuh experiment_sfu, 226-356): the same
 * flags, phase order, completion epochs and JSONL records, emitted one line
 * per callback.  Returns 0, or 1 with the reason in pm_last_error() (a record
 * may already have been emitted when a post-run check fails).
 */
typedef void (*pm_line_cb)(const char* line, void* user);
int pm_powerbench(int argc, const char* const* argv, pm_line_cb cb, void* user);

/*
 * One CTA of the tcgen05 tensor arm on its own: fills A (128 x 64) and
 * B (256 x 64) fp16 like the tensor workload does (seed, uniform[-1,1) when
 * `uniform`), runs `iterations` x 4 K-slices into accumulator 0 of
 * `accumulators` and copies accumulator 0 (128 x N fp32, N = 512/accumulators
 * rounded down to 16, at most 256) to `out`; optionally the operands too.
 * No counterpart in the reference: it checks the MMA path numerically.
 */
int pm_tensor_probe(int accumulators, uint64_t iterations, int uniform, uint64_t seed, float* out,
                    size_t out_count, uint16_t* a_out, uint16_t* b_out);

/*
 * The powerbench gemm arm's own cuBLAS call (cublasGemmEx, fp16 A and B,
 * fp32 C, column-major, the arm's operand fill; cuda/gpu_bench.cu:784-790 is
 * the reference's call) once on m x k by k x n (each 1..4096): C to `out`
 * (m * n floats, column-major), optionally the operands too.  It checks the
 * library comparison arm numerically.
 */
int pm_gemm_probe(int m, int n, int k, int uniform, uint64_t seed, float* out, uint16_t* a_out, uint16_t* b_out);

/*
 * pm_group_bootstrap_device for callers that cannot allocate device memory
 * (a process whose own pool owns the whole device, a runtime that forbids
 * foreign allocations, a service that must fix the library's footprint in
 * advance).  No counterpart in the reference.  It calls no cudaMalloc,
 * cudaFree or allocating library routine: the prepared histograms and index
 * streams live in one fixed array inside this library, of
 * pm_bootstrap_static_scratch_capacity() bytes (32 MiB), which every GPU that
 * loads the library holds until the process exits.  Every group's stream is
 * kept while they fit; beyond that, groups of up to seven members are drawn
 * without one.  A job needing more than the array even then (n_groups x 6864
 * bytes, plus n_groups x resamples x max_members bytes when max_members > 7)
 * is rejected with PM_E_LIMIT.  Inputs and outputs are the caller's device buffers, as for
 * pm_group_bootstrap_device; job->max_members must bound every group.
 * The first call on a device looks up the array's device address and uploads
 * the generator constants; make that first call before any stream capture.
 * All calls share the array (nothing in it needs to start at zero), so calls
 * whose kernels overlap on the GPU race: serialize them on one stream.
 */
size_t pm_bootstrap_static_scratch_capacity(void);
int pm_group_bootstrap_device_static(const pm_bootstrap_job* job, void* stream);

/*
 * The complete FP32 nonlinear functions of the powerbench
 * exp|tanh|silu|rmsnorm|softmax workloads on caller device buffers (the
 * reference's cuda/nonlinear.cuh: init_nonlinear 5-14, pointwise_nonlinear_kernel
 * 23-38, row_nonlinear_kernel 59-89, launched as gpu_bench.cu:796-801).
 * pm_nonlinear_fill_device writes n inputs ((int(w & 0xffff) - 32768) / 8192 +
 * shift) or, with gamma != 0, RMSNorm weights (0.75 + (w & 0xffff) / 131072),
 * w = splitmix64 finaliser of (i ^ seed) truncated to 32 bits.
 * pm_nonlinear_apply_device applies `function` `iterations` times to n inputs
 * on a blocks x threads grid (softmax/RMSNorm: rows of row_width, one row per
 * block, grid-stride over rows; pointwise: row_width 0).  Buffers are 16-byte
 * aligned; gamma (row_width floats) is read by RMSNorm only.
 */
enum { PM_NL_EXP = 0, PM_NL_TANH = 1, PM_NL_SILU = 2, PM_NL_SOFTMAX = 3, PM_NL_RMSNORM = 4 };
int pm_nonlinear_fill_device(float* data, uint64_t n, uint64_t seed, float shift, int gamma, void* stream);
int pm_nonlinear_apply_device(int32_t function, const float* input, const float* gamma, float* output, uint64_t n,
                              int32_t row_width, uint64_t iterations, int32_t blocks, int32_t threads, void* stream);

/* Raw resample index stream of random.Random(seed).choices(range(n), k=n),
 * repeated `resamples` times: out[r*n + j] (host buffer). Pins the generator. */
int pm_resample_indices(uint64_t seed, int32_t n, int32_t resamples, int32_t* out);

#ifdef __cplusplus
}
#endif
#endif /* PMB200_H */
