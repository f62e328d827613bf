// Refcounted paged-KV block allocator with a radix prefix index (C++ hot path of
// the scheduler).  Semantics match kapsl_sdk_b200.llm.block_manager.BlockAllocator:
//   * free list with lowest-id-first reuse;
//   * blocks whose refcount drops to 0 but that name a cached prefix stay
//     reusable ("cached free") until evicted: lowest priority first (the
//     highest priority of the sequences that committed or reused the block),
//     then LRU by last release or FIFO by id;
//   * prefix match over full blocks, capped at len-1 tokens so the last token is
//     always recomputed.
// Reference: crates/kapsl-llm/src/block_manager.rs:5-277, kv_cache.rs:640-696,
// 1107-1154, 1250-1308, radix_tree.rs:1-112.
#pragma once

#include <stdint.h>

#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

namespace kapsl {

struct OutOfBlocksError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

struct VecHash {
  size_t operator()(const std::vector<int32_t>& v) const noexcept {
    uint64_t h = 1469598103934665603ull;
    for (int32_t x : v) {
      h ^= (uint32_t)x;
      h *= 1099511628211ull;
    }
    return (size_t)h;
  }
};

class BlockAllocator {
 public:
  BlockAllocator(int64_t num_blocks, int block_size, bool enable_prefix_cache, const std::string& eviction);

  int64_t num_blocks() const { return num_blocks_; }
  int block_size() const { return block_size_; }
  int64_t num_free() const { return (int64_t)free_list_.size() + (int64_t)cached_count_; }
  int64_t num_used() const { return num_blocks_ - num_free(); }
  double usage() const { return num_blocks_ ? (double)num_used() / (double)num_blocks_ : 0.0; }
  uint64_t evicted_blocks() const { return evicted_; }
  int refcount(int64_t b) const { return ref_.at(b); }

  std::vector<int64_t> allocate(int64_t n);
  void incref(const std::vector<int64_t>& blocks);
  void free(const std::vector<int64_t>& blocks);
  std::vector<int64_t> match_prefix(const std::vector<int32_t>& tokens);
  void commit_prefix(const std::vector<int32_t>& tokens, const std::vector<int64_t>& blocks, int priority = 0);
  bool is_cached(int64_t b) const { return by_block_[b] != nullptr; }

 private:
  struct Node {
    int64_t block = -1;
    Node* parent = nullptr;
    std::vector<int32_t> key;
    std::unordered_map<std::vector<int32_t>, std::unique_ptr<Node>, VecHash> children;
  };
  void remove_block_node(int64_t b);
  void cached_push(int64_t b);
  void cached_erase(int64_t b);
  int64_t cached_pop();

  int64_t num_blocks_;
  int block_size_;
  bool prefix_;
  bool lru_;
  std::vector<int> ref_;
  std::vector<int64_t> free_list_;  // back() = next to hand out
  // cached-free blocks ordered by (priority, release tick or block id)
  using Key = std::tuple<int, uint64_t, int64_t>;
  std::set<Key> cached_;
  std::vector<Key> cached_key_;
  std::vector<uint8_t> in_cached_;
  std::vector<int> prio_;
  uint64_t tick_ = 0;
  size_t cached_count_ = 0;
  uint64_t evicted_ = 0;
  Node root_;
  std::vector<Node*> by_block_;
};

}  // namespace kapsl
