// Bounded work queue of the runtime scheduler (one per executor worker): an
// overflow policy on put, micro-batch takes (up to max items within a delay),
// in-flight accounting for the queue depth, close.  Reference:
// crates/kapsl-scheduler/src/gpu_executor.rs:11-329 and scheduler.rs:14-410.
//
// Jobs are opaque Python objects held by reference (PyObject*, one reference per
// queued job).  Waiting happens on a std::condition_variable with the GIL
// released, and the queue mutex is never held while the GIL is being acquired:
// a call takes its Python references with the GIL, releases it, works on the
// deque under the mutex, and only then takes the GIL back.
#pragma once

#include <Python.h>

#include <chrono>
#include <condition_variable>
#include <cstddef>
#include <deque>
#include <mutex>
#include <vector>

namespace kapsl {

class WorkQueue {
 public:
  enum Policy { kBlock = 0, kDropNewest = 1, kDropOldest = 2 };
  enum Put { kRejected = 0, kAccepted = 1 };

  explicit WorkQueue(size_t capacity) : cap_(capacity ? capacity : 1) {}
  // Destroyed by its Python owner, with the GIL held: drops the queued jobs' references.
  ~WorkQueue() {
    for (PyObject* p : q_) Py_XDECREF(p);
  }
  WorkQueue(const WorkQueue&) = delete;
  WorkQueue& operator=(const WorkQueue&) = delete;

  // Called without the GIL.  `job` carries a reference the queue now owns when
  // kAccepted; *dropped receives the reference of a job evicted by kDropOldest.
  int put(PyObject* job, int policy, bool block, PyObject** dropped) {
    *dropped = nullptr;
    std::unique_lock<std::mutex> lk(mu_);
    while (q_.size() >= cap_) {
      if (policy == kDropNewest || !block) return kRejected;
      if (policy == kDropOldest) {
        *dropped = q_.front();
        q_.pop_front();
        break;
      }
      cv_.wait_for(lk, std::chrono::milliseconds(50));
      if (closed_) return kRejected;
    }
    q_.push_back(job);
    cv_.notify_all();
    return kAccepted;
  }

  // Called without the GIL.  Waits (in 50 ms slices) for a first job, then
  // collects up to max_items until delay_s after the first; the returned
  // references are the caller's.  Empty when closed and drained.
  std::vector<PyObject*> take(size_t max_items, double delay_s) {
    std::vector<PyObject*> out;
    std::unique_lock<std::mutex> lk(mu_);
    while (q_.empty() && !closed_) cv_.wait_for(lk, std::chrono::milliseconds(50));
    if (q_.empty()) return out;
    out.push_back(q_.front());
    q_.pop_front();
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(delay_s);
    while (out.size() < max_items) {
      if (!q_.empty()) {
        out.push_back(q_.front());
        q_.pop_front();
        continue;
      }
      if (closed_ || cv_.wait_until(lk, deadline) == std::cv_status::timeout) {
        while (out.size() < max_items && !q_.empty()) {
          out.push_back(q_.front());
          q_.pop_front();
        }
        break;
      }
    }
    in_flight_ += out.size();
    cv_.notify_all();
    return out;
  }

  void done(size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    in_flight_ -= n < in_flight_ ? n : in_flight_;
    cv_.notify_all();
  }
  void close() {
    std::lock_guard<std::mutex> g(mu_);
    closed_ = true;
    cv_.notify_all();
  }
  size_t depth() {
    std::lock_guard<std::mutex> g(mu_);
    return q_.size() + in_flight_;
  }
  bool closed() {
    std::lock_guard<std::mutex> g(mu_);
    return closed_;
  }
  size_t capacity() const { return cap_; }
  // Jobs still queued (their references; used to release them at teardown).
  std::vector<PyObject*> drain() {
    std::lock_guard<std::mutex> g(mu_);
    std::vector<PyObject*> out(q_.begin(), q_.end());
    q_.clear();
    return out;
  }

 private:
  const size_t cap_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<PyObject*> q_;
  size_t in_flight_ = 0;
  bool closed_ = false;
};

}  // namespace kapsl
