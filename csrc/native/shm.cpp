#include "shm.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <memory>

namespace kapsl {
namespace shm {

static std::string os_name(const std::string& name) { return name.empty() || name[0] == '/' ? name : "/" + name; }

uint8_t dtype_code(const std::string& c) {
  if (c == "float64") return 1;
  if (c == "int32") return 2;
  if (c == "int64") return 3;
  return 0;
}
std::string dtype_from_code(uint8_t code) {
  switch (code) {
    case 1: return "float64";
    case 2: return "int32";
    case 3: return "int64";
    default: return "float32";
  }
}

Region Region::create(const std::string& name, size_t size) {
  if (size < TENSOR_POOL_OFFSET + 4096) throw std::invalid_argument("shm region too small");
  const std::string n = os_name(name);
  shm_unlink(n.c_str());
  int fd = shm_open(n.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  if (fd < 0) throw std::runtime_error("shm_open(" + n + ") failed: " + strerror(errno));
  if (ftruncate(fd, (off_t)size) != 0) {
    close(fd);
    shm_unlink(n.c_str());
    throw std::runtime_error("ftruncate failed: " + std::string(strerror(errno)));
  }
  void* p = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    shm_unlink(n.c_str());
    throw std::runtime_error("mmap failed: " + std::string(strerror(errno)));
  }
  Region r;
  r.base_ = static_cast<uint8_t*>(p);
  r.size_ = size;
  r.name_ = name;
  r.owner_ = true;
  if (pipe(r.fds_) == 0) {
    fcntl(r.fds_[0], F_SETFL, O_NONBLOCK);
    fcntl(r.fds_[1], F_SETFL, O_NONBLOCK);
  } else {
    r.fds_[0] = r.fds_[1] = -1;
  }
  ShmHeader h{MAGIC, VERSION, REQ_RING_OFFSET, RESP_RING_OFFSET, TENSOR_POOL_OFFSET, size - TENSOR_POOL_OFFSET,
              r.fds_[0], r.fds_[1]};
  std::memcpy(r.base_, &h, sizeof(h));
  return r;
}

Region Region::open(const std::string& name) {
  const std::string n = os_name(name);
  int fd = shm_open(n.c_str(), O_RDWR, 0600);
  if (fd < 0) throw std::runtime_error("cannot open shared memory '" + name + "': " + strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    throw std::runtime_error("fstat failed");
  }
  void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) throw std::runtime_error("mmap failed: " + std::string(strerror(errno)));
  Region r;
  r.base_ = static_cast<uint8_t*>(p);
  r.size_ = (size_t)st.st_size;
  r.name_ = name;
  const ShmHeader& h = r.header();
  if (r.size_ < sizeof(ShmHeader) || h.magic != MAGIC || h.version != VERSION)
    throw std::runtime_error("shared memory '" + name + "' has no kapsl header");
  return r;
}

Region::Region(Region&& o) noexcept { *this = std::move(o); }
Region& Region::operator=(Region&& o) noexcept {
  if (this != &o) {
    std::swap(base_, o.base_);
    std::swap(size_, o.size_);
    std::swap(name_, o.name_);
    std::swap(owner_, o.owner_);
    std::swap(fds_, o.fds_);
  }
  return *this;
}
Region::~Region() {
  if (base_) munmap(base_, size_);
  if (owner_) {
    shm_unlink(os_name(name_).c_str());
    if (fds_[0] >= 0) close(fds_[0]);
    if (fds_[1] >= 0) close(fds_[1]);
  }
}

// ------------------------------------------------------------- allocators
SlotAllocator::SlotAllocator(uint64_t base, uint64_t slot_size, uint64_t num_slots, double ttl_s)
    : base_(base), slot_(std::max<uint64_t>(slot_size, 1)), n_(std::max<uint64_t>(num_slots, 1)), ttl_s_(ttl_s) {
  leases_.resize(n_);
}

std::optional<uint64_t> SlotAllocator::try_allocate(uint64_t size, bool force) {
  if (size == 0 || size > slot_) return std::nullopt;
  std::lock_guard<std::mutex> g(mu_);
  const auto now = clock::now();
  uint64_t oldest = n_;
  for (uint64_t i = 0; i < n_; ++i) {
    const uint64_t s = (next_ + i) % n_;
    auto& l = leases_[s];
    const bool live = l.has_value() && std::chrono::duration<double>(now - *l).count() < ttl_s_;
    // a live lease on a guarded slot ends as soon as its reader has marked it read
    if (live && !(guard_ && unread_word(s).load(std::memory_order_acquire) == 0)) {
      if (!guard_ && (oldest == n_ || *l < *leases_[oldest])) oldest = s;
      continue;
    }
    l = now;
    next_ = (s + 1) % n_;
    if (guard_) unread_word(s).store(1, std::memory_order_release);
    return base_ + s * slot_;
  }
  if (force && oldest < n_) {  // never with a guard: an unread result is not overwritten
    leases_[oldest] = now;
    next_ = (oldest + 1) % n_;
    return base_ + oldest * slot_;
  }
  return std::nullopt;
}

bool SlotAllocator::release(uint64_t offset) {
  if (offset < base_ || offset >= base_ + n_ * slot_ || (offset - base_) % slot_ != 0) return false;
  std::lock_guard<std::mutex> g(mu_);
  leases_[(offset - base_) / slot_].reset();
  return true;
}

size_t SlotAllocator::in_use() const {
  std::lock_guard<std::mutex> g(mu_);
  const auto now = clock::now();
  size_t c = 0;
  for (const auto& l : leases_)
    if (l.has_value() && std::chrono::duration<double>(now - *l).count() < ttl_s_) ++c;
  return c;
}

double SlotAllocator::oldest_lease_ms() const {
  std::lock_guard<std::mutex> g(mu_);
  const auto now = clock::now();
  double m = 0;
  for (const auto& l : leases_)
    if (l.has_value()) m = std::max(m, std::chrono::duration<double, std::milli>(now - *l).count());
  return m;
}

TieredAllocator::TieredAllocator(uint64_t base, uint64_t pool_bytes, const std::vector<uint64_t>& class_sizes,
                                 const std::vector<uint32_t>& weights, double ttl_s) {
  std::vector<uint64_t> sizes = class_sizes;
  if (sizes.empty()) sizes = {256ull << 10, 1ull << 20, 4ull << 20, 16ull << 20, 64ull << 20};
  std::vector<uint32_t> w = weights;
  w.resize(sizes.size(), 1);
  std::vector<size_t> order(sizes.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return sizes[a] < sizes[b]; });
  // one slot per class when it fits, then the rest split by weight share
  std::vector<uint64_t> nslots(sizes.size(), 0);
  uint64_t remaining = pool_bytes;
  for (size_t i : order)
    if (remaining >= sizes[i]) {
      nslots[i] = 1;
      remaining -= sizes[i];
    }
  uint64_t wsum = 0;
  for (size_t i : order)
    if (nslots[i]) wsum += w[i];
  if (wsum > 0) {
    const uint64_t budget = remaining;
    for (size_t i : order) {
      if (!nslots[i]) continue;
      const uint64_t share = budget / wsum * w[i];
      const uint64_t extra = std::min<uint64_t>(share, remaining) / sizes[i];
      nslots[i] += extra;
      remaining -= extra * sizes[i];
    }
    // leftover bytes go to the smallest classes that still fit
    for (size_t i : order)
      while (nslots[i] && remaining >= sizes[i]) {
        ++nslots[i];
        remaining -= sizes[i];
      }
  }
  uint64_t cursor = base;
  for (size_t i : order) {
    if (!nslots[i]) continue;
    classes_.push_back(std::make_unique<SlotAllocator>(cursor, sizes[i], nslots[i], ttl_s));
    cursor += nslots[i] * sizes[i];
  }
  if (classes_.empty()) classes_.push_back(std::make_unique<SlotAllocator>(base, std::max<uint64_t>(pool_bytes, 1), 1, ttl_s));
}

std::optional<uint64_t> TieredAllocator::try_allocate(uint64_t size, bool force) {
  for (auto& c : classes_)
    if (c->slot_size() >= size)
      if (auto o = c->try_allocate(size)) return o;
  if (force)
    for (auto& c : classes_)
      if (c->slot_size() >= size)
        if (auto o = c->try_allocate(size, true)) return o;
  return std::nullopt;
}
bool TieredAllocator::release(uint64_t offset) {
  for (auto& c : classes_)
    if (c->release(offset)) return true;
  return false;
}
size_t TieredAllocator::in_use() const {
  size_t n = 0;
  for (auto& c : classes_) n += c->in_use();
  return n;
}
double TieredAllocator::oldest_lease_ms() const {
  double m = 0;
  for (auto& c : classes_) m = std::max(m, c->oldest_lease_ms());
  return m;
}
uint64_t TieredAllocator::largest_slot() const {
  uint64_t m = 0;
  for (auto& c : classes_) m = std::max(m, c->slot_size());
  return m;
}
std::string TieredAllocator::layout_summary() const {
  std::string s;
  for (auto& c : classes_) {
    if (!s.empty()) s += ",";
    s += std::to_string(c->slot_size()) + "x" + std::to_string(c->num_slots());
  }
  return s;
}

// ------------------------------------------------------- per-model pools
ModelPools::ModelPools(uint64_t base, uint64_t total_bytes, const std::vector<ModelPoolSpec>& models, double ttl_s) {
  const uint64_t end = base + total_bytes;
  uint64_t cursor = base;
  for (const auto& m : models) {
    const uint64_t bytes = std::min<uint64_t>(m.pool_bytes, end - cursor);
    if (bytes == 0 || pools_.count(m.model_id)) continue;
    pools_[m.model_id] = Pool{cursor, cursor + bytes,
                              std::make_unique<TieredAllocator>(cursor, bytes, m.class_sizes, m.weights, ttl_s)};
    cursor += bytes;
  }
  shared_ = Pool{cursor, end, std::make_unique<TieredAllocator>(cursor, std::max<uint64_t>(end - cursor, 1),
                                                                std::vector<uint64_t>{}, std::vector<uint32_t>{}, ttl_s)};
}

std::optional<uint64_t> ModelPools::try_allocate(uint32_t model_id, uint64_t size, bool force) {
  auto it = pools_.find(model_id);
  TieredAllocator* own = it != pools_.end() ? it->second.alloc.get() : nullptr;
  TieredAllocator* shared = shared_.end != shared_.base ? shared_.alloc.get() : nullptr;
  for (int f = 0; f <= (force ? 1 : 0); ++f) {
    if (own)
      if (auto o = own->try_allocate(size, f == 1)) return o;
    if (shared)
      if (auto o = shared->try_allocate(size, f == 1)) return o;
  }
  return std::nullopt;
}

bool ModelPools::release(uint64_t offset) {
  for (auto& [id, p] : pools_)
    if (offset >= p.base && offset < p.end) return p.alloc->release(offset);
  if (offset >= shared_.base && offset < shared_.end) return shared_.alloc->release(offset);
  return false;
}

static PoolUsage usage_of(const TieredAllocator& a) { return PoolUsage{a.in_use(), a.oldest_lease_ms()}; }

PoolUsage ModelPools::model_usage(uint32_t model_id) const {
  auto it = pools_.find(model_id);
  return it == pools_.end() ? PoolUsage{} : usage_of(*it->second.alloc);
}
PoolUsage ModelPools::shared_usage() const {
  return shared_.end == shared_.base ? PoolUsage{} : usage_of(*shared_.alloc);
}
PoolUsage ModelPools::total_usage() const {
  PoolUsage t = shared_usage();
  for (auto& [id, p] : pools_) {
    const PoolUsage u = usage_of(*p.alloc);
    t.in_use += u.in_use;
    t.oldest_lease_ms = std::max(t.oldest_lease_ms, u.oldest_lease_ms);
  }
  return t;
}

std::pair<uint64_t, uint64_t> ModelPools::range(uint32_t model_id) const {
  if (model_id == UINT32_MAX) return {shared_.base, shared_.end};
  auto it = pools_.find(model_id);
  if (it == pools_.end()) return {0, 0};
  return {it->second.base, it->second.end};
}

std::string ModelPools::layout_summary() const {
  std::string s;
  for (auto& [id, p] : pools_) s += "model " + std::to_string(id) + ": " + p.alloc->layout_summary() + "; ";
  s += "shared: " + (shared_.end == shared_.base ? std::string("none") : shared_.alloc->layout_summary());
  return s;
}

std::vector<std::pair<uint32_t, uint64_t>> ModelPools::plan(uint64_t total_bytes,
                                                            std::vector<std::pair<uint32_t, uint32_t>> weights,
                                                            uint32_t reserve_pct, uint64_t min_pool) {
  std::sort(weights.begin(), weights.end());
  uint64_t wsum = 0;
  for (auto& w : weights) {
    w.second = std::clamp<uint32_t>(w.second, 1, 1000);
    wsum += w.second;
  }
  const uint64_t reserve = std::max<uint64_t>((uint64_t)((unsigned __int128)total_bytes * reserve_pct / 100), min_pool);
  const uint64_t avail = total_bytes > reserve ? total_bytes - reserve : 0;
  std::vector<std::pair<uint32_t, uint64_t>> out;
  uint64_t given = 0;
  for (size_t i = 0; i < weights.size(); ++i) {
    const uint64_t bytes = i + 1 == weights.size()
                               ? avail - std::min(given, avail)
                               : (uint64_t)((unsigned __int128)avail * weights[i].second / std::max<uint64_t>(wsum, 1));
    if (bytes < min_pool) continue;
    out.emplace_back(weights[i].first, bytes);
    given += bytes;
  }
  return out;
}

// ------------------------------------------------------------ shared leases
static uint64_t monotonic_ms() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000ull + (uint64_t)ts.tv_nsec / 1000000ull;
}

SharedLeases::SharedLeases(Region& r, uint64_t base, uint64_t bytes, double ttl_s)
    : layout_(base, bytes), ttl_s_(ttl_s) {
  words_ = reinterpret_cast<std::atomic<uint64_t>*>(r.base() + kWordsOffset);
}

std::optional<uint64_t> SharedLeases::try_allocate(uint64_t size) {
  size_t word = 0;
  const uint64_t now = monotonic_ms();
  const uint64_t expiry = now + (uint64_t)(ttl_s_ * 1000.0);
  for (const auto& c : layout_.classes()) {
    const size_t first = word;
    word += c->num_slots();
    if (c->slot_size() < size) continue;
    for (uint64_t s = 0; s < c->num_slots() && first + s < kMaxWords; ++s) {
      std::atomic<uint64_t>& w = words_[first + s];
      uint64_t cur = w.load(std::memory_order_acquire);
      if (cur != 0 && cur > now) continue;  // leased and not expired
      if (w.compare_exchange_strong(cur, expiry, std::memory_order_acq_rel)) return c->base() + s * c->slot_size();
    }
  }
  return std::nullopt;
}

bool SharedLeases::release(uint64_t offset) {
  size_t word = 0;
  for (const auto& c : layout_.classes()) {
    if (offset >= c->base() && offset < c->base() + c->num_slots() * c->slot_size()) {
      const uint64_t s = (offset - c->base()) / c->slot_size();
      if (word + s >= kMaxWords) return false;
      words_[word + s].store(0, std::memory_order_release);
      return true;
    }
    word += c->num_slots();
  }
  return false;
}

// ----------------------------------------------------------------- tensors
uint64_t tensor_bytes(const wire::Packet& p) { return sizeof(TensorHeader) + p.data.size(); }

void mark_result_read(Region& r, uint64_t off) {
  if (off < kResultGuard || (off - kResultGuard) % 8 != 0 || !r.in_bounds(off - kResultGuard, 8)) return;
  reinterpret_cast<std::atomic<uint64_t>*>(r.base() + off - kResultGuard)->store(0, std::memory_order_release);
}

void write_tensor(Region& r, uint64_t off, const wire::Packet& p) {
  if (p.shape.size() > 8) throw std::invalid_argument("at most 8 dimensions fit a TensorHeader");
  if (!r.in_bounds(off, tensor_bytes(p))) throw std::out_of_range("tensor does not fit the shared memory region");
  TensorHeader h;
  std::memset(&h, 0, sizeof(h));
  h.ndim = (uint32_t)p.shape.size();
  h.dtype = dtype_code(p.dtype);
  for (size_t i = 0; i < p.shape.size(); ++i) h.shape[i] = p.shape[i];
  h.data_size = p.data.size();
  std::memcpy(r.base() + off, &h, sizeof(h));
  std::memcpy(r.base() + off + sizeof(h), p.data.data(), p.data.size());
}

wire::Packet read_tensor(const Region& r, uint64_t off) {
  if (!r.in_bounds(off, sizeof(TensorHeader))) throw std::out_of_range("tensor offset outside the shared memory region");
  TensorHeader h;
  std::memcpy(&h, r.base() + off, sizeof(h));
  if (h.ndim > 8) throw std::out_of_range("tensor header has more than 8 dimensions");
  if (!r.in_bounds(off + sizeof(h), h.data_size)) throw std::out_of_range("tensor data outside the shared memory region");
  wire::Packet p;
  p.shape.assign(h.shape, h.shape + h.ndim);
  p.dtype = dtype_from_code(h.dtype);
  p.data.assign(reinterpret_cast<const char*>(r.base() + off + sizeof(h)), (size_t)h.data_size);
  return p;
}

void write_error(Region& r, uint64_t off, const std::string& msg) {
  if (!r.in_bounds(off, 8 + msg.size())) throw std::out_of_range("error blob does not fit");
  const uint64_t n = msg.size();
  std::memcpy(r.base() + off, &n, 8);
  std::memcpy(r.base() + off + 8, msg.data(), n);
}

std::string read_error(const Region& r, uint64_t off) {
  if (!r.in_bounds(off, 8)) throw std::out_of_range("error offset outside the region");
  uint64_t n;
  std::memcpy(&n, r.base() + off, 8);
  if (!r.in_bounds(off + 8, n)) throw std::out_of_range("error blob outside the region");
  return std::string(reinterpret_cast<const char*>(r.base() + off + 8), (size_t)n);
}

}  // namespace shm
}  // namespace kapsl
