/*
 * libpmb200 — the sharded summarize's row exchange over NVLink peer memory.
 *
 * summarize (powermodeling/analysis.py:1400-1470) needs every trial's metric
 * row before any group is bootstrapped, and a group's repeats may have been
 * analysed on other ranks.  One process per GPU: each rank analyses its
 * slice of the trials, and the analysis kernel itself stores every trial's
 * metric row and valid flag into the gathered row buffer of every rank
 * (peer pointers from CUDA IPC), so the exchange overlaps the analysis of
 * the remaining trials instead of following it.  The last CTA of a launch
 * then raises this rank's arrival flag on every rank; pm_peer_wait_device
 * holds a stream until every rank's flag has reached the step's epoch.
 * Every wait is bounded: on expiry it records an error and returns.
 *
 * Conventions as in pmb200.h.  Pointers in pm_peer_rows are device pointers
 * valid on the calling rank (its own buffers, or peers' buffers opened with
 * pm_peer_open).
 */
#ifndef PMB200_PEER_H
#define PMB200_PEER_H

#include <stddef.h>
#include <stdint.h>

#include "pmb200.h"

#ifdef __cplusplus
extern "C" {
#endif

#define PM_MAX_RANKS 8

/* A CUDA IPC handle of a device allocation made by pm_peer_alloc. */
typedef struct pm_peer_handle {
  unsigned char bytes[64];
} pm_peer_handle;

/* Device memory (zero-filled) that other ranks may open; *handle receives its
 * IPC handle.  Free with pm_peer_free. */
int pm_peer_alloc(size_t bytes, void** device_ptr, pm_peer_handle* handle);
int pm_peer_free(void* device_ptr);

/* Map another rank's pm_peer_alloc buffer into this process (peer access
 * over NVLink); release with pm_peer_close. */
int pm_peer_open(const pm_peer_handle* handle, void** device_ptr);
int pm_peer_close(void* device_ptr);

/* Where an analysis launch on rank `rank` delivers its rows. */
typedef struct pm_peer_rows {
  int32_t n_ranks;                    /* 1..PM_MAX_RANKS */
  int32_t rank;                       /* this rank */
  int32_t row_offset;                 /* global row of this launch's first trial */
  uint32_t epoch;                     /* > the previous launch's epoch */
  double* metrics[PM_MAX_RANKS];      /* each rank's gathered rows [total_rows * PM_N_METRICS] */
  uint8_t* valid[PM_MAX_RANKS];       /* each rank's gathered valid flags [total_rows] */
  uint32_t* flags[PM_MAX_RANKS];      /* each rank's arrival flags [n_ranks]; this rank sets entry `rank` */
  uint32_t* done;                     /* this rank's CTA counter (pm_peer_alloc, 4 bytes, starts at 0) */
} pm_peer_rows;

/* pm_analyze_trials_device, plus every trial's metric row and valid flag
 * stored at row row_offset + trial of every rank's gathered buffers, and
 * this rank's flag raised to `epoch` on every rank once the launch's rows
 * are all out.  Launches on one rank must use increasing epochs and the
 * same trial count (the counter target is epoch * n_trials). */
int pm_analyze_trials_device_exchange(const pm_trials* trials, const pm_policy* policy, pm_trial_results* out,
                                      void* scratch, size_t scratch_bytes, const pm_peer_rows* rows, void* stream);

/* Where a bootstrap finish on rank `rank` delivers its groups: each
 * receiving rank's gathered buffer is [n_ranks][3][per_rank][n_metrics]
 * (medians, interval lows, interval highs), this rank's local group j going
 * to [rank][k][j].  root < 0: every rank receives (an all-gather); root >= 0:
 * only rank `root` does (a gather), and out[r] / flags[r] of the other ranks
 * may be NULL. */
typedef struct pm_peer_groups {
  int32_t n_ranks;                    /* 1..PM_MAX_RANKS */
  int32_t rank;                       /* this rank */
  int32_t per_rank;                   /* group stride: groups owned per rank (>= this launch's n_groups) */
  uint32_t epoch;                     /* > the previous launch's epoch */
  double* out[PM_MAX_RANKS];          /* each receiving rank's gathered group buffer */
  uint32_t* flags[PM_MAX_RANKS];      /* each receiving rank's arrival flags [n_ranks]; this rank sets entry `rank` */
  uint32_t* done;                     /* this rank's CTA counter (starts at 0) */
  int32_t root;                       /* -1: all-gather; 0..n_ranks-1: gather to that rank only */
} pm_peer_groups;

/* pm_bootstrap_finish_device, plus every group's medians and interval ends
 * stored into every receiving rank's gathered buffer, and this rank's flag
 * raised to `epoch` on every receiving rank once they are all out (at once
 * when this rank owns no group).  Same epoch rules as
 * pm_analyze_trials_device_exchange, with the group count in place of the
 * trial count. */
int pm_bootstrap_finish_device_exchange(const pm_bootstrap_job* job, void* scratch, size_t scratch_bytes,
                                        const pm_peer_groups* groups, void* stream);

/* Hold `stream` until flags[0..n_ranks) all reach `epoch` (a one-CTA kernel
 * polling at system scope).  If that takes longer than timeout_ms, the
 * kernel stores 1 into *error (device memory) and returns. */
int pm_peer_wait_device(const uint32_t* flags, int32_t n_ranks, uint32_t epoch, uint32_t timeout_ms, int32_t* error,
                        void* stream);

/* A device-side start line for all ranks: store `epoch` into entry `rank` of
 * every rank's flag array (flags[r], n_ranks entries each, system-scope
 * release stores), then hold `stream` until this rank's own array
 * (flags[rank]) has every entry at `epoch` or beyond.  Ranks whose hosts
 * enqueue work after it at different moments start that work together on
 * their GPUs.  The wait is bounded like pm_peer_wait_device's. */
int pm_peer_gate_device(uint32_t* const* flags, int32_t n_ranks, int32_t rank, uint32_t epoch, uint32_t timeout_ms,
                        int32_t* error, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PMB200_PEER_H */
