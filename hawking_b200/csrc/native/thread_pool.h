// Minimal persistent fork-join pool for the CPU reference (row-parallel matvecs, quantisers).
#pragma once
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace hk {

class ThreadPool {
 public:
  explicit ThreadPool(int n) : n_(n < 1 ? 1 : n) {
    for (int i = 1; i < n_; ++i) workers_.emplace_back([this, i] { loop(i); });
  }
  ~ThreadPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return n_; }
  // Run fn(begin, end) over [0, n) split into size() contiguous chunks; blocks until done.
  void parallel_for(size_t n, const std::function<void(size_t, size_t)>& fn) {
    if (n_ == 1 || n < 2) { fn(0, n); return; }
    {
      std::lock_guard<std::mutex> g(mu_);
      job_ = &fn;
      total_ = n;
      pending_ = n_ - 1;
      ++gen_;
    }
    cv_.notify_all();
    run_chunk(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void run_chunk(int i) {
    size_t per = (total_ + n_ - 1) / n_;
    size_t a = i * per, e = a + per < total_ ? a + per : total_;
    if (a < e) (*job_)(a, e);
  }
  void loop(int i) {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return gen_ != seen; });
      seen = gen_;
      if (stop_) return;
      lk.unlock();
      run_chunk(i);
      lk.lock();
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }
  int n_;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t, size_t)>* job_ = nullptr;
  size_t total_ = 0;
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

}  // namespace hk
