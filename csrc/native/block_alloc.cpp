#include "block_alloc.h"

#include <algorithm>

namespace kapsl {

BlockAllocator::BlockAllocator(int64_t num_blocks, int block_size, bool enable_prefix_cache,
                               const std::string& eviction)
    : num_blocks_(num_blocks), block_size_(block_size), prefix_(enable_prefix_cache), lru_(eviction != "fifo") {
  if (num_blocks <= 0 || block_size <= 0) throw std::invalid_argument("num_blocks and block_size must be > 0");
  if (eviction != "lru" && eviction != "fifo") throw std::invalid_argument("eviction must be 'lru' or 'fifo'");
  ref_.assign(num_blocks, 0);
  free_list_.reserve(num_blocks);
  for (int64_t b = num_blocks - 1; b >= 0; --b) free_list_.push_back(b);
  cached_key_.resize(num_blocks);
  in_cached_.assign(num_blocks, 0);
  prio_.assign(num_blocks, 0);
  by_block_.assign(num_blocks, nullptr);
}

void BlockAllocator::cached_push(int64_t b) {
  in_cached_[b] = 1;
  ++cached_count_;
  cached_key_[b] = Key{prio_[b], lru_ ? tick_++ : (uint64_t)b, b};
  cached_.insert(cached_key_[b]);
}

void BlockAllocator::cached_erase(int64_t b) {
  if (!in_cached_[b]) return;
  in_cached_[b] = 0;
  --cached_count_;
  cached_.erase(cached_key_[b]);
}

int64_t BlockAllocator::cached_pop() {
  const int64_t b = std::get<2>(*cached_.begin());
  cached_erase(b);
  return b;
}

void BlockAllocator::remove_block_node(int64_t b) {
  Node* n = by_block_[b];
  if (!n) return;
  // unregister the whole subtree, then detach it from its parent
  std::vector<Node*> stack{n};
  while (!stack.empty()) {
    Node* x = stack.back();
    stack.pop_back();
    if (x->block >= 0) {
      by_block_[x->block] = nullptr;
      prio_[x->block] = 0;
      // descendants are unreachable now: unused ones go back to the plain free list
      if (x->block != b && in_cached_[x->block]) {
        cached_erase(x->block);
        free_list_.push_back(x->block);
      }
    }
    for (auto& kv : x->children) stack.push_back(kv.second.get());
  }
  if (n->parent) n->parent->children.erase(n->key);  // frees the subtree
}

std::vector<int64_t> BlockAllocator::allocate(int64_t n) {
  if (n < 0) throw std::invalid_argument("negative block count");
  if (n > num_free())
    throw OutOfBlocksError("need " + std::to_string(n) + " blocks, " + std::to_string(num_free()) + " free");
  std::vector<int64_t> out;
  out.reserve(n);
  for (int64_t i = 0; i < n; ++i) {
    int64_t b;
    if (!free_list_.empty()) {
      b = free_list_.back();
      free_list_.pop_back();
    } else {
      b = cached_pop();
      remove_block_node(b);
      ++evicted_;
    }
    ref_[b] = 1;
    out.push_back(b);
  }
  return out;
}

void BlockAllocator::incref(const std::vector<int64_t>& blocks) {
  for (int64_t b : blocks) {
    if (b < 0 || b >= num_blocks_) throw std::out_of_range("block id out of range");
    if (ref_[b] == 0) cached_erase(b);
    ++ref_[b];
  }
}

void BlockAllocator::free(const std::vector<int64_t>& blocks) {
  for (auto it = blocks.rbegin(); it != blocks.rend(); ++it) {
    const int64_t b = *it;
    if (b < 0 || b >= num_blocks_) throw std::out_of_range("block id out of range");
    if (ref_[b] <= 0) throw std::runtime_error("double free of block " + std::to_string(b));
    if (--ref_[b] == 0) {
      if (prefix_ && by_block_[b] != nullptr)
        cached_push(b);
      else
        free_list_.push_back(b);
    }
  }
}

std::vector<int64_t> BlockAllocator::match_prefix(const std::vector<int32_t>& tokens) {
  std::vector<int64_t> out;
  if (!prefix_ || tokens.size() <= 1) return out;
  const size_t usable = tokens.size() - 1;
  Node* node = &root_;
  std::vector<int32_t> key(block_size_);
  for (size_t i = 0; i + block_size_ <= usable; i += block_size_) {
    std::copy(tokens.begin() + i, tokens.begin() + i + block_size_, key.begin());
    auto it = node->children.find(key);
    if (it == node->children.end()) break;
    node = it->second.get();
    out.push_back(node->block);
  }
  incref(out);
  return out;
}

void BlockAllocator::commit_prefix(const std::vector<int32_t>& tokens, const std::vector<int64_t>& blocks,
                                   int priority) {
  if (!prefix_) return;
  Node* node = &root_;
  const size_t nfull = std::min(tokens.size() / block_size_, blocks.size());
  for (size_t i = 0; i < nfull; ++i) {
    std::vector<int32_t> key(tokens.begin() + i * block_size_, tokens.begin() + (i + 1) * block_size_);
    auto it = node->children.find(key);
    if (it == node->children.end()) {
      const int64_t b = blocks[i];
      if (by_block_[b] != nullptr) return;  // block already names another prefix
      auto child = std::make_unique<Node>();
      child->block = b;
      child->parent = node;
      child->key = key;
      Node* raw = child.get();
      node->children.emplace(std::move(key), std::move(child));
      by_block_[b] = raw;
      node = raw;
    } else {
      node = it->second.get();
    }
    prio_[node->block] = std::max(prio_[node->block], priority);
  }
}

}  // namespace kapsl
