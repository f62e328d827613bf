#include "hnsw.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <queue>
#include <stdexcept>
#include <thread>

#ifdef __AVX2__
#include <immintrin.h>
#endif

namespace kapsl {
namespace rag {

namespace {

// Visited marks without clearing: a per-thread array of epochs.
struct Visited {
  std::vector<uint32_t> mark;
  uint32_t epoch = 0;
  void reset(size_t n) {
    if (mark.size() < n) mark.resize(n, 0);
    if (++epoch == 0) {  // wrapped: clear once
      std::fill(mark.begin(), mark.end(), 0);
      epoch = 1;
    }
  }
  bool test_and_set(int32_t i) {
    if (mark[i] == epoch) return true;
    mark[i] = epoch;
    return false;
  }
};

Visited& visited() {
  static thread_local Visited v;
  return v;
}

}  // namespace

Hnsw::Hnsw(int dim, int M, int ef_construction, uint64_t seed)
    : dim_(dim), M_(M), M0_(2 * M), efc_(ef_construction), ml_(1.0 / std::log((double)std::max(M, 2))), rng_(seed) {
  if (dim <= 0 || M < 2 || ef_construction < 1) throw std::invalid_argument("hnsw: bad dim / M / ef_construction");
}

float Hnsw::dist(const float* a, int32_t b) const {
  const float* v = vec(b);
  int i = 0;
  float s = 0.f;
#ifdef __AVX2__
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  for (; i + 16 <= dim_; i += 16) {
    acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(v + i), acc0);
    acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(v + i + 8), acc1);
  }
  const __m256 acc = _mm256_add_ps(acc0, acc1);
  const __m128 h = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
  const __m128 h2 = _mm_add_ps(h, _mm_movehl_ps(h, h));
  s = _mm_cvtss_f32(_mm_add_ss(h2, _mm_shuffle_ps(h2, h2, 1)));
#endif
  for (; i < dim_; ++i) s += a[i] * v[i];
  return 1.f - s;
}

void Hnsw::neighbours(int32_t n, int level, std::vector<int32_t>& out) const {
  if (concurrent_) {
    std::lock_guard<std::mutex> g(node_mu_[n]);
    out = links_[n][level];
  } else {
    out = links_[n][level];
  }
}

int32_t Hnsw::greedy(const float* q, int32_t ep, int level) const {
  float d = dist(q, ep);
  std::vector<int32_t> nb;
  for (bool moved = true; moved;) {
    moved = false;
    neighbours(ep, level, nb);
    for (int32_t n : nb) {
      const float dn = dist(q, n);
      if (dn < d) {
        d = dn;
        ep = n;
        moved = true;
      }
    }
  }
  return ep;
}

std::vector<Hnsw::Cand> Hnsw::beam(const float* q, int32_t ep, int ef, int level) const {
  Visited& vis = visited();
  vis.reset(links_.size());
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> frontier;  // nearest on top
  std::priority_queue<Cand> best;                                             // farthest on top
  const float d0 = dist(q, ep);
  vis.test_and_set(ep);
  frontier.push({d0, ep});
  best.push({d0, ep});
  std::vector<int32_t> nb;
  while (!frontier.empty()) {
    const Cand c = frontier.top();
    if (c.first > best.top().first && (int)best.size() >= ef) break;
    frontier.pop();
    neighbours(c.second, level, nb);
    for (int32_t n : nb) {
      if (vis.test_and_set(n)) continue;
      const float dn = dist(q, n);
      if ((int)best.size() < ef || dn < best.top().first) {
        frontier.push({dn, n});
        best.push({dn, n});
        if ((int)best.size() > ef) best.pop();
      }
    }
  }
  std::vector<Cand> out(best.size());
  for (size_t i = out.size(); i-- > 0;) {
    out[i] = best.top();
    best.pop();
  }
  return out;
}

std::vector<int32_t> Hnsw::select(std::vector<Cand> cand, int m) const {
  std::sort(cand.begin(), cand.end());
  std::vector<int32_t> kept;
  for (const Cand& c : cand) {
    if ((int)kept.size() >= m) break;
    bool good = true;
    for (int32_t r : kept)
      if (dist(vec(c.second), r) < c.first) {
        good = false;
        break;
      }
    if (good) kept.push_back(c.second);
  }
  // fill up with the nearest discarded ones so sparse regions keep degree
  for (const Cand& c : cand) {
    if ((int)kept.size() >= m) break;
    if (std::find(kept.begin(), kept.end(), c.second) == kept.end()) kept.push_back(c.second);
  }
  return kept;
}

int64_t Hnsw::append(const float* in, int level) {
  const int32_t id = (int32_t)links_.size();
  double norm = 0.0;
  for (int i = 0; i < dim_; ++i) norm += (double)in[i] * in[i];
  const float inv = norm > 0.0 ? (float)(1.0 / std::sqrt(norm)) : 0.f;
  for (int i = 0; i < dim_; ++i) data_.push_back(in[i] * inv);
  links_.emplace_back(level + 1);
  removed_.push_back(0);
  node_mu_.emplace_back();
  return id;
}

void Hnsw::link(int32_t id) {
  const float* q = vec(id);
  const int level = (int)links_[id].size() - 1;
  int32_t ep;
  int top;
  {
    std::lock_guard<std::mutex> g(entry_mu_);
    if (entry_ < 0) {
      entry_ = id;
      top_ = level;
      return;
    }
    ep = entry_;
    top = top_;
  }
  for (int l = top; l > level; --l) ep = greedy(q, ep, l);
  for (int l = std::min(level, top); l >= 0; --l) {
    std::vector<Cand> w = beam(q, ep, efc_, l);
    const int mmax = l == 0 ? M0_ : M_;
    const std::vector<int32_t> mine = select(w, M_);
    {
      std::unique_lock<std::mutex> g(node_mu_[id], std::defer_lock);
      if (concurrent_) g.lock();
      links(id, l) = mine;
    }
    for (int32_t n : mine) {
      std::unique_lock<std::mutex> g(node_mu_[n], std::defer_lock);
      if (concurrent_) g.lock();
      std::vector<int32_t>& nl = links(n, l);
      nl.push_back(id);
      if ((int)nl.size() > mmax) {
        std::vector<Cand> c;
        c.reserve(nl.size());
        for (int32_t x : nl) c.push_back({dist(vec(n), x), x});
        nl = select(std::move(c), mmax);
      }
    }
    ep = w.front().second;
  }
  std::lock_guard<std::mutex> g(entry_mu_);
  if (level > top_) {
    top_ = level;
    entry_ = id;
  }
}

int64_t Hnsw::add(const float* in) {
  std::lock_guard<std::mutex> turn(turn_);
  std::unique_lock<std::shared_mutex> lock(mu_);
  std::uniform_real_distribution<double> u(std::nextafter(0.0, 1.0), 1.0);
  const int64_t id = append(in, (int)std::floor(-std::log(u(rng_)) * ml_));
  link((int32_t)id);
  return id;
}

int64_t Hnsw::add_batch(const float* vecs, int64_t n, int threads) {
  std::lock_guard<std::mutex> turn(turn_);
  std::unique_lock<std::shared_mutex> lock(mu_);
  const int64_t first = (int64_t)links_.size();
  if (n <= 0) return first;
  std::uniform_real_distribution<double> u(std::nextafter(0.0, 1.0), 1.0);
  data_.reserve(data_.size() + (size_t)n * dim_);
  for (int64_t i = 0; i < n; ++i) append(vecs + i * dim_, (int)std::floor(-std::log(u(rng_)) * ml_));
  int64_t start = first;
  for (; start < first + n && (entry_ < 0 || start - first < 64); ++start) link((int32_t)start);  // seed serially
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  threads = (int)std::min<int64_t>(threads, first + n - start);
  if (threads <= 1) {
    for (int64_t i = start; i < first + n; ++i) link((int32_t)i);
    return first;
  }
  concurrent_ = true;
  std::atomic<int64_t> next{start};
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&] {
      for (int64_t i; (i = next.fetch_add(1)) < first + n;) link((int32_t)i);
    });
  for (auto& t : pool) t.join();
  concurrent_ = false;
  return first;
}

void Hnsw::remove(int64_t label) {
  std::lock_guard<std::mutex> turn(turn_);
  std::unique_lock<std::shared_mutex> lock(mu_);
  if (label >= 0 && label < (int64_t)removed_.size()) removed_[label] = 1;
}

Hnsw::Hnsw(Hnsw&& o) noexcept
    : dim_(o.dim_), M_(o.M_), M0_(o.M0_), efc_(o.efc_), ml_(o.ml_), rng_(o.rng_), data_(std::move(o.data_)),
      links_(std::move(o.links_)), removed_(std::move(o.removed_)), entry_(o.entry_), top_(o.top_) {
  for (size_t i = 0; i < links_.size(); ++i) node_mu_.emplace_back();
}

void Hnsw::save(const std::string& path) const {
  std::shared_lock<std::shared_mutex> lock(mu_);
  std::FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw std::runtime_error("hnsw.save: cannot open " + path);
  bool ok = true;
  auto put = [&](const void* p, size_t n) { ok = ok && (n == 0 || std::fwrite(p, 1, n, f) == n); };  // empty lists may have no buffer
  const int32_t head[5] = {dim_, M_, efc_, entry_, top_};
  const int64_t n = (int64_t)links_.size();
  put("KHNSW001", 8);
  put(head, sizeof(head));
  put(&n, 8);
  put(data_.data(), data_.size() * sizeof(float));
  put(removed_.data(), removed_.size());
  for (const auto& levels : links_) {
    const int32_t nl = (int32_t)levels.size();
    put(&nl, 4);
    for (const auto& l : levels) {
      const int32_t c = (int32_t)l.size();
      put(&c, 4);
      put(l.data(), l.size() * 4);
    }
  }
  ok = (std::fclose(f) == 0) && ok;
  if (!ok) throw std::runtime_error("hnsw.save: write failed for " + path);
}

Hnsw Hnsw::load(const std::string& path) {
  std::FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) throw std::runtime_error("hnsw.load: cannot open " + path);
  auto fail = [&](const char* what) {
    std::fclose(f);
    throw std::runtime_error(std::string("hnsw.load: ") + what + " in " + path);
  };
  auto get = [&](void* p, size_t n) {
    if (n != 0 && std::fread(p, 1, n, f) != n) fail("truncated file");
  };
  char magic[8];
  int32_t head[5];
  int64_t n;
  get(magic, 8);
  get(head, sizeof(head));
  get(&n, 8);
  if (std::memcmp(magic, "KHNSW001", 8) != 0 || head[0] <= 0 || head[0] > (1 << 16) || head[1] < 2 ||
      head[1] > 1024 || head[2] < 1 || n < 0 || n > ((int64_t)1 << 31) - 1 || head[3] < -1 || head[3] >= n ||
      head[4] < -1 || head[4] > 64)
    fail("bad header");
  Hnsw h(head[0], head[1], head[2]);
  h.entry_ = head[3];
  h.top_ = head[4];
  // read the payload in bounded pieces so a forged count cannot demand a huge buffer up front
  std::vector<float> vecs;
  std::vector<uint8_t> removed;
  for (int64_t i = 0; i < n; ++i) {
    const size_t at = vecs.size();
    vecs.resize(at + (size_t)h.dim_);
    get(vecs.data() + at, (size_t)h.dim_ * sizeof(float));
  }
  removed.resize((size_t)n);
  get(removed.data(), removed.size());
  h.data_ = std::move(vecs);
  h.removed_ = std::move(removed);
  h.links_.resize((size_t)n);
  for (int64_t i = 0; i < n; ++i) {
    int32_t nl;
    get(&nl, 4);
    if (nl < 1 || nl > 65) fail("bad level count");
    h.links_[i].resize(nl);
    for (auto& l : h.links_[i]) {
      int32_t c;
      get(&c, 4);
      if (c < 0 || c > 2 * h.M0_) fail("bad neighbour count");
      l.resize(c);
      get(l.data(), (size_t)c * 4);
    }
  }
  std::fclose(f);
  for (int64_t i = 0; i < n; ++i)  // every id must name a node that has the level it is linked at
    for (size_t lv = 0; lv < h.links_[i].size(); ++lv)
      for (int32_t x : h.links_[i][lv])
        if (x < 0 || x >= n || h.links_[x].size() <= lv) throw std::runtime_error("hnsw.load: bad link in " + path);
  if (n > 0 && (h.entry_ < 0 || (int)h.links_[h.entry_].size() != h.top_ + 1))
    throw std::runtime_error("hnsw.load: bad entry point in " + path);
  if (n == 0 && (h.entry_ != -1 || h.top_ != -1)) throw std::runtime_error("hnsw.load: bad entry point in " + path);
  for (int64_t i = 0; i < n; ++i) h.node_mu_.emplace_back();
  return h;
}

int64_t Hnsw::size() const {
  std::shared_lock<std::shared_mutex> lock(mu_);
  return (int64_t)links_.size();
}

std::vector<std::pair<float, int64_t>> Hnsw::search(const float* qin, int k, int ef, const uint8_t* allowed,
                                                    int64_t allowed_len) const {
  { std::lock_guard<std::mutex> turn(turn_); }  // wait behind a writer that is queued
  std::shared_lock<std::shared_mutex> lock(mu_);
  std::vector<std::pair<float, int64_t>> out;
  if (entry_ < 0 || k <= 0) return out;
  std::vector<float> q(qin, qin + dim_);
  double norm = 0.0;
  for (float v : q) norm += (double)v * v;
  if (norm == 0.0) return out;
  const float inv = (float)(1.0 / std::sqrt(norm));
  for (float& v : q) v *= inv;
  int32_t ep = entry_;
  for (int l = top_; l > 0; --l) ep = greedy(q.data(), ep, l);
  for (const Cand& c : beam(q.data(), ep, std::max(ef, k), 0)) {
    if (removed_[c.second]) continue;
    if (allowed && (c.second >= allowed_len || !allowed[c.second])) continue;
    out.push_back({1.f - c.first, c.second});
    if ((int)out.size() >= k) break;
  }
  return out;
}

}  // namespace rag
}  // namespace kapsl
