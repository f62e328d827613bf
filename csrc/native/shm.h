// Shared-memory transport: region layout, MPMC ring, tensor headers and slot
// allocators.  Byte layout follows crates/kapsl-shm/src/memory.rs:4-118,
// ring_buffer.rs:21-229 and server.rs:52-69:
//
//   offset 0       ShmHeader (48 B): magic "AIMO" 0x41494D4F, version 1,
//                  request ring @4096, response ring @69632, tensor pool
//                  @131072, max_tensor_size = size - 131072, notify fds
//   offset 4096    Ring<ShmRequest>  (capacity argument 1024)
//   offset 69632   Ring<ShmResponse> (capacity argument 1024)
//   offset 131072  tensor pool: TensorHeader (80 B) + data; error blobs are
//                  [u64 len][utf8]
//
// Ring: the first three T-sized slots hold head_reserved, head_committed and
// tail (each an atomic size_t at the slot start); data slots follow; indices
// wrap modulo (capacity - 3); one slot stays empty.  Producers reserve with a
// CAS on head_reserved, write, then publish in reservation order with a CAS on
// head_committed.  Consumers copy the slot and then CAS the tail (the copy is
// taken before the slot is released, so a fast producer cannot overwrite it).
// The indices wrap, so a thread stalled between reading an index and its CAS
// for a full turn of the ring would succeed on a stale value (ABA).  To rule
// that out, this library's producers and consumers each take a side lock
// first: 8-byte words at byte 8 of the head_reserved slot (producers) and of
// the tail slot (consumers), bytes that the index layout leaves unused.  A
// lock word holds the holder's CLOCK_MONOTONIC time in ns (shifted left 10,
// low bits a per-thread tag); a holder older than one second is presumed dead
// and its lock is taken over.
#pragma once

#include <stdint.h>

#include <atomic>
#include <chrono>
#include <functional>
#include <memory>
#include <map>
#include <mutex>
#include <optional>
#include <string>
#include <thread>
#include <vector>

#include "wire.h"

namespace kapsl {
namespace shm {

constexpr uint32_t MAGIC = 0x41494D4F;
constexpr uint32_t VERSION = 1;
constexpr uint64_t REQ_RING_OFFSET = 4096;
constexpr uint64_t RESP_RING_OFFSET = 4096 + 64 * 1024;
constexpr uint64_t TENSOR_POOL_OFFSET = 128 * 1024;
constexpr size_t RING_CAPACITY_ARG = 1024;

struct ShmHeader {
  uint32_t magic;
  uint32_t version;
  uint64_t request_queue_offset;
  uint64_t response_queue_offset;
  uint64_t tensor_pool_offset;
  uint64_t max_tensor_size;
  int32_t notify_read_fd;
  int32_t notify_write_fd;
};
static_assert(sizeof(ShmHeader) == 48, "ShmHeader is 48 bytes");

struct TensorHeader {
  uint32_t ndim;
  uint8_t dtype;  // 0 f32, 1 f64, 2 i32, 3 i64 (others are written as 0)
  uint8_t pad[3];
  int64_t shape[8];
  uint64_t data_size;
};
static_assert(sizeof(TensorHeader) == 80, "TensorHeader is 80 bytes");

struct ShmRequest {
  wire::TransportRequestMeta meta;
  uint64_t tensor_offset;
  uint64_t tensor_size;
};
static_assert(sizeof(ShmRequest) == 40, "ShmRequest is 40 bytes");

struct ShmResponse {
  wire::TransportResponseMeta meta;
  uint64_t result_offset;
  uint64_t result_size;
  uint64_t error_offset;  // 0 = no error
};
static_assert(sizeof(ShmResponse) == 48, "ShmResponse is 48 bytes");

uint8_t dtype_code(const std::string& canonical);
std::string dtype_from_code(uint8_t code);

class Region {
 public:
  // Create (and own) a region; an existing object of that name is replaced.
  static Region create(const std::string& name, size_t size);
  static Region open(const std::string& name);
  Region() = default;
  Region(Region&& o) noexcept;
  Region& operator=(Region&& o) noexcept;
  Region(const Region&) = delete;
  ~Region();

  uint8_t* base() const { return base_; }
  size_t size() const { return size_; }
  const ShmHeader& header() const { return *reinterpret_cast<const ShmHeader*>(base_); }
  const std::string& name() const { return name_; }
  bool owner() const { return owner_; }
  // Every offset/size coming from a peer is checked against the mapping.
  bool in_bounds(uint64_t off, uint64_t len) const { return off <= size_ && len <= size_ - off; }

 private:
  uint8_t* base_ = nullptr;
  size_t size_ = 0;
  std::string name_;
  bool owner_ = false;
  int fds_[2] = {-1, -1};
};

template <class T>
class Ring {
 public:
  static_assert(sizeof(T) >= 2 * sizeof(std::atomic<size_t>), "slot must hold an index and a lock word");
  Ring(uint8_t* at, size_t capacity_arg, bool init) : slots_(reinterpret_cast<T*>(at)), cap_(capacity_arg - 3) {
    if (init) {
      new (&idx(0)) std::atomic<size_t>(0);
      new (&idx(1)) std::atomic<size_t>(0);
      new (&idx(2)) std::atomic<size_t>(0);
      new (&lock_word(0)) std::atomic<uint64_t>(0);
      new (&lock_word(2)) std::atomic<uint64_t>(0);
    }
  }
  bool push(const T& item) {
    SideLock g(lock_word(0));
    if (!g.held) return false;  // another producer holds the lock; the caller retries like on a full ring
    for (;;) {
      size_t reserved = idx(0).load(std::memory_order_relaxed);
      size_t next = (reserved + 1) % cap_;
      if (next == idx(2).load(std::memory_order_acquire)) return false;  // full
      if (idx(0).compare_exchange_weak(reserved, next, std::memory_order_relaxed)) {
        slots_[3 + reserved] = item;
        size_t expect = reserved;
        unsigned spins = 0;
        while (!idx(1).compare_exchange_weak(expect, next, std::memory_order_release, std::memory_order_relaxed)) {
          expect = reserved;
          if ((++spins & 63) == 0) std::this_thread::yield();
        }
        return true;
      }
    }
  }
  std::optional<T> pop() {
    SideLock g(lock_word(2));
    if (!g.held) return std::nullopt;
    for (;;) {
      size_t tail = idx(2).load(std::memory_order_relaxed);
      size_t committed = idx(1).load(std::memory_order_acquire);
      if (tail == committed) return std::nullopt;
      T item = slots_[3 + tail];
      size_t next = (tail + 1) % cap_;
      if (idx(2).compare_exchange_weak(tail, next, std::memory_order_release, std::memory_order_relaxed)) return item;
    }
  }
  size_t len() const {
    size_t c = idx(1).load(std::memory_order_acquire), t = idx(2).load(std::memory_order_acquire);
    return c >= t ? c - t : cap_ - t + c;
  }
  size_t capacity() const { return cap_ - 1; }

 private:
  // Held for a slot copy and two index updates.  Waits up to ~2 ms for the
  // lock (then reports it not held, which callers treat like an empty or full
  // ring and retry); takes over a lock whose holder stamped it more than one
  // second ago.
  struct SideLock {
    std::atomic<uint64_t>& w;
    uint64_t token = 0;
    bool held = false;
    explicit SideLock(std::atomic<uint64_t>& word) : w(word) {
      static thread_local const uint64_t tag =
          (std::hash<std::thread::id>{}(std::this_thread::get_id()) & 1023) | 1;
      for (unsigned spins = 0; spins < 20000; ++spins) {
        const uint64_t now = now_ns();
        token = (now << 10) | tag;
        uint64_t cur = w.load(std::memory_order_relaxed);
        if (cur == 0 || (now > (cur >> 10) && now - (cur >> 10) > 1000000000ull)) {
          if (w.compare_exchange_strong(cur, token, std::memory_order_acquire, std::memory_order_relaxed)) {
            held = true;
            return;
          }
        }
        if ((spins & 15) == 15) std::this_thread::yield();
      }
    }
    ~SideLock() {
      if (!held) return;
      uint64_t expect = token;
      w.compare_exchange_strong(expect, 0, std::memory_order_release, std::memory_order_relaxed);
    }
    static uint64_t now_ns() {
      return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                 std::chrono::steady_clock::now().time_since_epoch())
          .count();
    }
  };
  std::atomic<size_t>& idx(int i) const { return *reinterpret_cast<std::atomic<size_t>*>(&slots_[i]); }
  std::atomic<uint64_t>& lock_word(int i) const {
    return *reinterpret_cast<std::atomic<uint64_t>*>(reinterpret_cast<uint8_t*>(&slots_[i]) + 8);
  }
  T* slots_;
  size_t cap_;
};

// Result slots handed to clients start with a kResultGuard-byte header whose first
// 64-bit word is 1 while the result is unread; the client stores 0 after copying
// it out (mark_result_read), and the tensor itself starts kResultGuard bytes in.
constexpr uint64_t kResultGuard = 64;

// Round-robin slot allocator with TTL leases (expired leases are reclaimed).
class SlotAllocator {
 public:
  SlotAllocator(uint64_t base, uint64_t slot_size, uint64_t num_slots, double ttl_s = 30.0);
  // force: when every slot is leased, take over the one leased longest ago.  With a
  // guard set, a slot whose unread word is 0 is free again before its lease expires,
  // taking a slot sets the word to 1, and force never takes over an unread result.
  std::optional<uint64_t> try_allocate(uint64_t size, bool force = false);
  void set_guard(uint8_t* region_base) { guard_ = region_base; }
  bool release(uint64_t offset);
  size_t in_use() const;
  double oldest_lease_ms() const;
  uint64_t slot_size() const { return slot_; }
  uint64_t num_slots() const { return n_; }
  uint64_t base() const { return base_; }

 private:
  using clock = std::chrono::steady_clock;
  uint64_t base_, slot_, n_;
  double ttl_s_;
  mutable std::mutex mu_;
  std::vector<std::optional<clock::time_point>> leases_;
  uint64_t next_ = 0;
  uint8_t* guard_ = nullptr;
  std::atomic<uint64_t>& unread_word(uint64_t s) const {
    return *reinterpret_cast<std::atomic<uint64_t>*>(guard_ + base_ + s * slot_);
  }
};

// Size classes 256 KiB, 1 MiB, 4 MiB, 16 MiB, 64 MiB (smallest fitting class
// first, then larger ones).  Bytes are split across classes in proportion to
// their weights, each class getting at least one slot when it fits.
class TieredAllocator {
 public:
  TieredAllocator(uint64_t base, uint64_t pool_bytes, const std::vector<uint64_t>& class_sizes = {},
                  const std::vector<uint32_t>& weights = {}, double ttl_s = 30.0);
  std::optional<uint64_t> try_allocate(uint64_t size, bool force = false);
  bool release(uint64_t offset);
  size_t in_use() const;
  double oldest_lease_ms() const;
  uint64_t largest_slot() const;
  std::string layout_summary() const;
  const std::vector<std::unique_ptr<SlotAllocator>>& classes() const { return classes_; }
  void set_guard(uint8_t* region_base) {
    for (auto& c : classes_) c->set_guard(region_base);
  }

 private:
  std::vector<std::unique_ptr<SlotAllocator>> classes_;
};

// Per-model sub-pools carved from one contiguous range: each model gets its own
// TieredAllocator over [cursor, cursor + pool_bytes) in the order given, and
// the bytes left over form a shared overflow pool with the default classes.
// An allocation tries the model's pool first, then the shared pool (unknown
// model ids go straight to the shared pool); a release finds its pool by
// offset range.  Reference: crates/kapsl-shm/src/allocator.rs:436-560
// (per-model allocator) and crates/kapsl-shm/src/server.rs:241-300 (sizing).
struct ModelPoolSpec {
  uint32_t model_id;
  uint64_t pool_bytes;
  std::vector<uint64_t> class_sizes;  // empty: default classes
  std::vector<uint32_t> weights;
};

struct PoolUsage {
  size_t in_use = 0;
  double oldest_lease_ms = 0;
};

class ModelPools {
 public:
  ModelPools(uint64_t base, uint64_t total_bytes, const std::vector<ModelPoolSpec>& models, double ttl_s = 30.0);
  // force: when both pools are full, take over the oldest lease (model pool first)
  std::optional<uint64_t> try_allocate(uint32_t model_id, uint64_t size, bool force = false);
  bool release(uint64_t offset);
  PoolUsage model_usage(uint32_t model_id) const;  // zeros when the model has no pool
  PoolUsage shared_usage() const;
  PoolUsage total_usage() const;
  bool has_pool(uint32_t model_id) const { return pools_.count(model_id) != 0; }
  // (base, end) of a model's pool, or of the shared pool for model_id == UINT32_MAX
  std::pair<uint64_t, uint64_t> range(uint32_t model_id) const;
  std::string layout_summary() const;
  void set_guard(uint8_t* region_base) {
    for (auto& [id, p] : pools_) p.alloc->set_guard(region_base);
    shared_.alloc->set_guard(region_base);
  }

  // Pool sizes for models weighted by expected concurrency: a reserve of
  // reserve_pct percent (at least min_pool bytes) stays shared, the rest is
  // split by weight (clamped to [1, 1000]) over models in id order, the last
  // taking the rounding remainder; slices under min_pool bytes are dropped
  // (those models use the shared pool).
  static std::vector<std::pair<uint32_t, uint64_t>> plan(uint64_t total_bytes,
                                                         std::vector<std::pair<uint32_t, uint32_t>> weights,
                                                         uint32_t reserve_pct = 10, uint64_t min_pool = 64 << 10);

 private:
  struct Pool {
    uint64_t base, end;
    std::unique_ptr<TieredAllocator> alloc;
  };
  std::map<uint32_t, Pool> pools_;
  Pool shared_;
};

// Slot leases shared by every client process of one region.  The slot layout
// is the TieredAllocator's over [base, base + bytes); each slot has one 64-bit
// lease word (0 = free, else the CLOCK_MONOTONIC expiry in ms) stored in the
// unused tail of header page 0 (offset 64, up to 500 words), taken with a CAS.
class SharedLeases {
 public:
  static constexpr uint64_t kWordsOffset = 64;
  static constexpr size_t kMaxWords = 500;
  SharedLeases(Region& r, uint64_t base, uint64_t bytes, double ttl_s = 30.0);
  std::optional<uint64_t> try_allocate(uint64_t size);
  bool release(uint64_t offset);
  uint64_t largest_slot() const { return layout_.largest_slot(); }
  std::string layout_summary() const { return layout_.layout_summary(); }

 private:
  TieredAllocator layout_;
  std::atomic<uint64_t>* words_;
  double ttl_s_;
};

// Tensor (header + data) helpers; return false / throw on out-of-bounds input.
void write_tensor(Region& r, uint64_t off, const wire::Packet& p);
wire::Packet read_tensor(const Region& r, uint64_t off);
void write_error(Region& r, uint64_t off, const std::string& msg);
// Client side of the result guard: the result (or error) at `off` has been copied out.
void mark_result_read(Region& r, uint64_t off);
std::string read_error(const Region& r, uint64_t off);
uint64_t tensor_bytes(const wire::Packet& p);

}  // namespace shm
}  // namespace kapsl
