// Approximate nearest-neighbour index for the RAG vector store: a
// Hierarchical Navigable Small World graph (Malkov and Yashunin, "Efficient
// and robust approximate nearest neighbor search using Hierarchical Navigable
// Small World graphs", TPAMI 2018) over cosine similarity.  Vectors are
// L2-normalised on insertion, so similarity is a dot product and distance is
// 1 - dot.
//
// * insert: a random level ~ floor(-ln U / ln M); greedy descent from the entry
//   point to that level, then per level a beam search of ef_construction and
//   neighbour selection by the paper's heuristic (a candidate is kept when it
//   is closer to the new node than to every neighbour kept so far), links made
//   both ways and over-full lists re-pruned with the same heuristic.
// * search: greedy descent to level 0, then a beam of max(ef, k).  `allowed`
//   (one byte per label, optional) filters what is returned, not what is
//   traversed, so the graph stays connected under any filter; removed labels
//   are traversed and never returned.
// Readers share a lock; insert and remove take it exclusively.  A batch insert
// links nodes from several threads under per-node locks.  A writer first
// takes a turnstile mutex that arriving readers also pass through, so a steady
// stream of searches cannot starve inserts (glibc's reader-writer lock prefers
// readers).
//
// The reference scores every stored row per query and leaves an ANN index as
// a to-do (crates/kapsl-rag/src/vector/mod.rs:26-359).
#pragma once

#include <stdint.h>

#include <deque>
#include <mutex>
#include <random>
#include <shared_mutex>
#include <string>
#include <utility>
#include <vector>

namespace kapsl {
namespace rag {

class Hnsw {
 public:
  Hnsw(int dim, int M = 16, int ef_construction = 200, uint64_t seed = 42);
  Hnsw(Hnsw&& o) noexcept;
  // Labels are dense: label i is the i-th inserted vector.  Returns it.
  int64_t add(const float* vec);
  // Inserts n vectors (row-major [n, dim]) with `threads` workers (0 = one per
  // core); returns the first label.  Levels are drawn in label order, so only
  // the links depend on the workers' interleaving.
  int64_t add_batch(const float* vecs, int64_t n, int threads = 0);
  void remove(int64_t label);
  // (similarity, label) best first; at most k.
  std::vector<std::pair<float, int64_t>> search(const float* q, int k, int ef, const uint8_t* allowed,
                                                int64_t allowed_len) const;
  int64_t size() const;
  int dim() const { return dim_; }
  // Binary file: "KHNSW001", dim, M, ef_construction, entry, top level, node
  // count, unit vectors, removed flags, then per node its level count and per
  // level its neighbour count and ids.  load() checks every count and id
  // against the file and throws on anything out of range.
  void save(const std::string& path) const;
  static Hnsw load(const std::string& path);

 private:
  using Cand = std::pair<float, int32_t>;  // (distance, node)
  float dist(const float* a, int32_t b) const;
  const float* vec(int32_t n) const { return data_.data() + (size_t)n * dim_; }
  int32_t greedy(const float* q, int32_t ep, int level) const;
  std::vector<Cand> beam(const float* q, int32_t ep, int ef, int level) const;  // nearest first
  std::vector<int32_t> select(std::vector<Cand> cand, int m) const;  // the paper's heuristic
  std::vector<int32_t>& links(int32_t n, int level) { return links_[n][level]; }
  // list of node n at `level`, copied under the node's lock while a batch
  // insert runs (workers update lists concurrently)
  void neighbours(int32_t n, int level, std::vector<int32_t>& out) const;
  int64_t append(const float* vec, int level);  // storage for one node, not linked
  void link(int32_t id);                        // connect a stored node into the graph

  int dim_, M_, M0_, efc_;
  double ml_;
  std::mt19937_64 rng_;
  std::vector<float> data_;
  std::vector<std::vector<std::vector<int32_t>>> links_;  // [node][level] -> neighbours
  std::vector<uint8_t> removed_;
  int32_t entry_ = -1;
  int top_ = -1;
  mutable std::shared_mutex mu_;
  mutable std::mutex turn_;
  mutable std::deque<std::mutex> node_mu_;  // per-node list locks (batch insert)
  std::mutex entry_mu_;                     // entry_ / top_ during a batch insert
  bool concurrent_ = false;
};

}  // namespace rag
}  // namespace kapsl
