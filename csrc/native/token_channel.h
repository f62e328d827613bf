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
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace kapsl {

class TokenChannel {
 public:
  enum Pop { kTokens = 0, kEnd = 1, kError = 2, kTimeout = 3 };

  void push(int32_t tok) {
    push_quiet(tok, false);
    wake();
  }
  // Appends a token (and, with `fin`, ends the stream) without waking the consumer;
  // the caller wakes it later with wake() (see TokenNotifier).
  void push_quiet(int32_t tok, bool fin) {
    std::lock_guard<std::mutex> g(mu_);
    if (closed_) return;
    q_.push_back(tok);
    if (fin) closed_ = true;
  }
  void wake() { cv_.notify_all(); }
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

// Wakes token-channel consumers off the producer's thread.  A condition-variable
// notify with a waiting consumer is a futex system call of a few microseconds;
// an engine step that feeds 256 streams paid ~1.6 ms for them on the engine loop's
// critical path.  The producer appends every token quietly and hands the batch of
// channels to this thread, which issues the wakeups while the next step runs.
// The thread lives for the rest of the process (never joined, so no exit-time
// ordering with the interpreter); channels stay alive through their shared_ptrs
// until woken.
class TokenNotifier {
 public:
  static TokenNotifier& get() {
    static TokenNotifier* n = new TokenNotifier();  // intentionally never destroyed
    return *n;
  }
  void post(std::vector<std::shared_ptr<TokenChannel>>&& batch) {
    if (batch.empty()) return;
    {
      std::lock_guard<std::mutex> g(mu_);
      pending_.push_back(std::move(batch));
    }
    cv_.notify_one();
  }

 private:
  TokenNotifier() { std::thread([this] { run(); }).detach(); }
  void run() {
    for (;;) {
      std::deque<std::vector<std::shared_ptr<TokenChannel>>> work;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return !pending_.empty(); });
        work.swap(pending_);
      }
      for (auto& batch : work)
        for (auto& c : batch) c->wake();
    }
  }
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<std::vector<std::shared_ptr<TokenChannel>>> pending_;
};

}  // namespace kapsl
