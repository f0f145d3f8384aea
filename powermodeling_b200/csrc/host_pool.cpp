#include "host_pool.h"

#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <mutex>
#include <thread>
#include <vector>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace pm {

HostBatch::HostBatch(size_t count, std::function<void(size_t)> fn)
    : task(std::move(fn)), n(count), flags(new std::atomic<unsigned char>[count ? count : 1]) {
  for (size_t i = 0; i < (count ? count : 1); ++i) flags[i].store(0, std::memory_order_relaxed);
}

namespace {

// Takes tasks from `b` until none is left; returns how many it ran.
size_t drain(HostBatch& b) {
  size_t ran = 0;
  for (;;) {
    const size_t i = b.next.fetch_add(1, std::memory_order_relaxed);
    if (i >= b.n) return ran;
    b.task(i);
    b.flags[i].store(1, std::memory_order_release);
    b.finished.fetch_add(1, std::memory_order_acq_rel);
    ++ran;
  }
}

// How long a worker keeps polling for the next batch before it sleeps:
// back-to-back calls then start without a thread wake-up.
// PM_HOST_SPIN_US overrides the default.
int spin_microseconds() {
  if (const char* env = std::getenv("PM_HOST_SPIN_US")) {
    const int v = std::atoi(env);
    return v < 0 ? 0 : v > 100000 ? 100000 : v;
  }
  return 500;
}

inline void cpu_relax() {
#if defined(__x86_64__)
  _mm_pause();
#else
  std::this_thread::yield();
#endif
}

class Pool {
 public:
  explicit Pool(int threads) : spin_(std::chrono::microseconds(spin_microseconds())) {
    for (int t = 0; t < threads; ++t) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(m_);
      quit_.store(true, std::memory_order_relaxed);
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
  }
  int size() const { return static_cast<int>(workers_.size()); }

  void run(HostBatch& b, const std::function<void()>& progress) {
    std::lock_guard<std::mutex> one_at_a_time(run_lock_);
    {
      std::lock_guard<std::mutex> g(m_);
      batch_ = &b;
      generation_.fetch_add(1, std::memory_order_release);
    }
    cv_.notify_all();
    for (;;) {
      const size_t i = b.next.fetch_add(1, std::memory_order_relaxed);
      if (i >= b.n) break;
      b.task(i);
      b.flags[i].store(1, std::memory_order_release);
      b.finished.fetch_add(1, std::memory_order_acq_rel);
      if (progress) progress();
    }
    while (b.finished.load(std::memory_order_acquire) < b.n) {
      if (progress) progress();
      std::this_thread::yield();
    }
    // Retire the batch: no worker may touch it after run returns.
    std::unique_lock<std::mutex> g(m_);
    batch_ = nullptr;
    idle_cv_.wait(g, [&] { return inside_ == 0; });
  }

 private:
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      // poll for a while before blocking (the lock and the condition decide)
      const auto until = std::chrono::steady_clock::now() + spin_;
      while (generation_.load(std::memory_order_acquire) == seen && !quit_.load(std::memory_order_relaxed) &&
             std::chrono::steady_clock::now() < until)
        cpu_relax();
      HostBatch* b = nullptr;
      {
        std::unique_lock<std::mutex> g(m_);
        cv_.wait(g, [&] { return quit_.load(std::memory_order_relaxed) || (generation_.load(std::memory_order_relaxed) != seen && batch_ != nullptr); });
        if (quit_.load(std::memory_order_relaxed)) return;
        seen = generation_.load(std::memory_order_relaxed);
        b = batch_;
        ++inside_;
      }
      drain(*b);
      {
        std::lock_guard<std::mutex> g(m_);
        --inside_;
      }
      idle_cv_.notify_all();
    }
  }

  std::vector<std::thread> workers_;
  std::mutex m_, run_lock_;
  std::condition_variable cv_, idle_cv_;
  HostBatch* batch_ = nullptr;
  std::atomic<uint64_t> generation_{0};
  int inside_ = 0;
  std::atomic<bool> quit_{false};
  const std::chrono::microseconds spin_;
};

int configured_threads() {
  if (const char* env = std::getenv("PM_HOST_THREADS")) {
    const int v = std::atoi(env);
    return v < 0 ? 0 : v > 64 ? 64 : v;
  }
  const unsigned hw = std::thread::hardware_concurrency();
  const int t = hw > 1 ? static_cast<int>(hw) - 1 : 0;
  return t > 3 ? 3 : t;   // host copies saturate memory bandwidth at about three threads
}

Pool& pool() {
  static Pool p(configured_threads());
  return p;
}

}  // namespace

void run_host_batch(HostBatch& batch, const std::function<void()>& progress) {
  if (batch.n == 0) {
    if (progress) progress();
    return;
  }
  pool().run(batch, progress);
}

int host_pool_threads() { return pool().size(); }

}  // namespace pm
