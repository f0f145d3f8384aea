// A fixed pool of host threads for staging work (copies into pinned memory,
// input validation), so a host-buffer entry point can overlap its copies
// with the DMA of what is already staged.
#pragma once
#include <atomic>
#include <cstddef>
#include <functional>
#include <memory>

namespace pm {

// One parallel loop: task(i) for i in [0, n), each exactly once; done(i)
// tells whether task i has finished.
struct HostBatch {
  std::function<void(size_t)> task;
  size_t n = 0;
  std::atomic<size_t> next{0};
  std::atomic<size_t> finished{0};
  std::unique_ptr<std::atomic<unsigned char>[]> flags;
  explicit HostBatch(size_t count, std::function<void(size_t)> fn);
  bool done(size_t i) const { return flags[i].load(std::memory_order_acquire) != 0; }
};

// Runs `batch` on the pool and on the calling thread.  The caller calls
// `progress` after each task it ran itself and while it waits, so it can
// act on finished tasks (start a DMA) before the whole batch ends; run
// returns after every task finished and no pool thread still holds the batch.
void run_host_batch(HostBatch& batch, const std::function<void()>& progress);

// Pool threads (not counting the caller); PM_HOST_THREADS overrides the
// default of min(3, hardware threads - 1).
int host_pool_threads();

}  // namespace pm
