// Token channel between the LLM engine loop and a streaming connection.
//
// The engine thread pushes each sampled token id of a request (one batched call
// per engine step for all requests); the server's connection thread pops them
// without holding the Python GIL and writes the stream frames itself.  A
// per-token Python generator on every connection thread made 256 concurrent
// streams contend for the GIL with the engine loop, capping a served decode at a
// few thousand tokens per second on the host; with the channel a token costs a
// mutex, a deque push and a condition-variable notify.
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <mutex>
#include <string>
#include <vector>

namespace kapsl {

class TokenChannel {
 public:
  enum Pop { kTokens = 0, kEnd = 1, kError = 2, kTimeout = 3 };

  void push(int32_t tok) {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (closed_) return;
      q_.push_back(tok);
    }
    cv_.notify_one();
  }
  void finish() { close(false, std::string()); }
  void fail(const std::string& msg) { close(true, msg); }
  // The consumer went away (the client closed its connection): the producer polls
  // this and aborts the request.
  void cancel() { cancelled_.store(true, std::memory_order_release); }
  bool cancelled() const { return cancelled_.load(std::memory_order_acquire); }

  // Waits up to timeout_ms for tokens or the end.  kTokens moves every queued token
  // into `out` (tokens queued before an end or error are always delivered first);
  // kEnd / kError once the queue is drained and the stream closed.
  int pop(std::vector<int32_t>& out, std::string& err, int timeout_ms) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return !q_.empty() || closed_; });
    if (!q_.empty()) {
      out.assign(q_.begin(), q_.end());
      q_.clear();
      return kTokens;
    }
    if (closed_) {
      err = err_;
      return failed_ ? kError : kEnd;
    }
    return kTimeout;
  }

 private:
  void close(bool failed, const std::string& msg) {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (closed_) return;
      closed_ = true;
      failed_ = failed;
      err_ = msg;
    }
    cv_.notify_all();
  }

  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<int32_t> q_;
  bool closed_ = false, failed_ = false;
  std::string err_;
  std::atomic<bool> cancelled_{false};
};

}  // namespace kapsl
