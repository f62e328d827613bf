"""Paged-KV block bookkeeping: refcounted allocator + radix prefix index.

Counterparts in the reference:
* ``BlockAllocator`` free list with LIFO reuse (crates/kapsl-llm/src/block_manager.rs:5-277),
* refcounted paged allocator, LRU/FIFO eviction of inactive blocks
  (crates/kapsl-llm/src/kv_cache.rs:640-696, 1107-1154),
* ``RadixTree`` over full blocks with prefix match capped at len-1 tokens
  (crates/kapsl-llm/src/radix_tree.rs:1-112, kv_cache.rs:1250-1308, 1375-1400).

Here the blocks index a GPU pool; the C++ allocator in ``kapsl_sdk_b200._native``
implements the same interface and is used when built (``NativeBlockAllocator``).
Freed blocks that hold a cached prefix stay reusable until evicted: lowest
priority first (the highest priority of the sequences that committed the
block; reference kv_cache.rs:1107-1154 orders inactive sequences the same
way), then LRU by last release or FIFO by block id.
"""
from __future__ import annotations

import itertools
from typing import Optional


class OutOfBlocks(RuntimeError):
    pass


class _RadixNode:
    __slots__ = ("children", "block", "parent", "key")

    def __init__(self, parent=None, key=None, block: int = -1):
        self.children: dict = {}
        self.block = block
        self.parent = parent
        self.key = key


class RadixPrefixIndex:
    """Trie keyed by full-block token tuples; each node names the block holding it."""

    def __init__(self, block_size: int):
        self.bs = block_size
        self.root = _RadixNode()
        self.by_block: dict[int, _RadixNode] = {}

    def match(self, tokens: list) -> list[int]:
        node, out = self.root, []
        for i in range(0, len(tokens) - self.bs + 1, self.bs):
            key = tuple(tokens[i:i + self.bs])
            child = node.children.get(key)
            if child is None:
                break
            out.append(child.block)
            node = child
        return out

    def insert(self, tokens: list, blocks: list[int]) -> list[int]:
        """Returns the blocks the index names along the path of ``tokens``."""
        node, path = self.root, []
        nfull = min(len(tokens) // self.bs, len(blocks))
        for i in range(nfull):
            key = tuple(tokens[i * self.bs:(i + 1) * self.bs])
            child = node.children.get(key)
            if child is None:
                if blocks[i] in self.by_block:  # block already names another prefix
                    break
                child = _RadixNode(node, key, blocks[i])
                node.children[key] = child
                self.by_block[blocks[i]] = child
            node = child
            path.append(child.block)
        return path

    def remove_block(self, block: int) -> list[int]:
        """Drop the node of ``block`` and its whole subtree; returns the blocks of
        the removed descendants (they are unreachable from now on)."""
        node = self.by_block.get(block)
        if node is None:
            return []
        stack = [node]
        gone = []
        while stack:
            n = stack.pop()
            self.by_block.pop(n.block, None)
            if n.block != block:
                gone.append(n.block)
            stack.extend(n.children.values())
        if node.parent is not None:
            node.parent.children.pop(node.key, None)
        return gone

    def __contains__(self, block: int) -> bool:
        return block in self.by_block


class BlockAllocator:
    """Refcounted allocator over ``num_blocks`` GPU pages with a prefix cache."""

    def __init__(self, num_blocks: int, block_size: int = 16, enable_prefix_cache: bool = True,
                 eviction: str = "lru"):
        assert eviction in ("lru", "fifo")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.enable_prefix_cache = enable_prefix_cache
        self.eviction = eviction
        self.ref = [0] * num_blocks
        self.free_list: list[int] = list(range(num_blocks - 1, -1, -1))  # pop() -> lowest id first
        self.cached_free: dict = {}  # refcount 0 but holding a prefix -> eviction key
        self.prio: dict = {}  # block -> highest priority of the sequences that committed it
        self.index = RadixPrefixIndex(block_size)
        self.evicted_blocks = 0
        self._tick = itertools.count()

    # ---------------------------------------------------------------- stats
    def num_free(self) -> int:
        return len(self.free_list) + len(self.cached_free)

    def num_used(self) -> int:
        return self.num_blocks - self.num_free()

    def usage(self) -> float:
        return self.num_used() / max(1, self.num_blocks)

    # ----------------------------------------------------------- alloc/free
    def allocate(self, n: int) -> list[int]:
        if n > self.num_free():
            raise OutOfBlocks(f"need {n} blocks, {self.num_free()} free")
        out = []
        for _ in range(n):
            if self.free_list:
                b = self.free_list.pop()
            else:
                b = min(self.cached_free, key=self.cached_free.__getitem__)
                del self.cached_free[b]
                self.prio.pop(b, None)
                for d in self.index.remove_block(b):
                    self.prio.pop(d, None)
                    if d in self.cached_free:  # unreachable cached descendants become plain free
                        del self.cached_free[d]
                        self.free_list.append(d)
                self.evicted_blocks += 1
            self.ref[b] = 1
            out.append(b)
        return out

    def incref(self, blocks: list[int]) -> None:
        for b in blocks:
            if self.ref[b] == 0:
                self.cached_free.pop(b, None)
            self.ref[b] += 1

    def free(self, blocks: list[int]) -> None:
        for b in reversed(blocks):
            r = self.ref[b] - 1
            if r < 0:
                raise RuntimeError(f"double free of block {b}")
            self.ref[b] = r
            if r == 0:
                if self.enable_prefix_cache and b in self.index:
                    # eviction order: lowest priority first, then LRU (release tick) or FIFO (id)
                    self.cached_free[b] = (self.prio.get(b, 0), next(self._tick) if self.eviction == "lru" else b)
                else:
                    self.free_list.append(b)

    # --------------------------------------------------------- prefix cache
    def match_prefix(self, tokens: list) -> list[int]:
        """Blocks holding the longest cached prefix of ``tokens``, capped so that
        at least the last token is recomputed; the blocks are increfed."""
        if not self.enable_prefix_cache or len(tokens) <= 1:
            return []
        blocks = self.index.match(tokens[:len(tokens) - 1])
        self.incref(blocks)
        return blocks

    def commit_prefix(self, tokens: list, blocks: list[int], priority: int = 0) -> None:
        """Register every full block of ``tokens`` (whose KV is computed); the
        blocks' eviction priority rises to ``priority``."""
        if self.enable_prefix_cache:
            for b in self.index.insert(tokens, blocks):
                self.prio[b] = max(self.prio.get(b, 0), priority)


def make_allocator(num_blocks: int, block_size: int = 16, enable_prefix_cache: bool = True,
                   eviction: str = "lru", prefer_native: bool = True):
    """The C++ allocator when the native module is built, else the Python one."""
    if prefer_native:
        try:
            from .._ext import native

            return native().BlockAllocator(num_blocks, block_size, enable_prefix_cache, eviction)
        except Exception:
            pass
    return BlockAllocator(num_blocks, block_size, enable_prefix_cache, eviction)
