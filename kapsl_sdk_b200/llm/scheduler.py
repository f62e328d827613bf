"""Continuous-batching scheduler with chunked prefill over the GPU block pool.

The reference ``LLMScheduler`` (crates/kapsl-llm/src/scheduler.rs:69-297)
admits a waiting request only if its *whole* prompt fits the token budget and
then runs every running group each step.  This scheduler keeps the same queue
structure (waiting / running, priority-ordered preemption, session groups keep
their blocks) and adds chunked prefill: each step has a budget of
``max_num_batched_tokens``; running decodes take one token each, then prompt
chunks fill the rest, so long prompts never stall decoding.

Preemption (the victim is the lowest-priority, latest-arrived running
sequence) either frees the victim's blocks and re-queues it for recomputation
("recompute"), or, with ``preemption="swap"``, moves the pages holding its
computed KV to host memory and parks it in the swapped queue ("swap", while
the host swap space has room).  Each step first swaps parked sequences back
in, oldest first, when their pages fit with one free block left per running
sequence (reference scheduler.rs:69-297: swap-in FIFO before admission).
The engine performs the page copies the batch lists (``swap_in`` before
``swap_out``, both before the step's kernels, on the same stream).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from .block_manager import OutOfBlocks
from .sequence import Sequence, SequenceStatus


@dataclass
class ScheduledBatch:
    decode: list = field(default_factory=list)    # sequences generating one token
    prefill: list = field(default_factory=list)   # (sequence, chunk_len)
    preempted: list = field(default_factory=list)
    preempted_slots: list = field(default_factory=list)  # their slots before preemption
    admitted: list = field(default_factory=list)  # moved from waiting/swapped to running this step
    swap_out: list = field(default_factory=list)  # (sequence, blocks to copy to host, in order)
    swap_in: list = field(default_factory=list)   # (sequence, blocks to restore into)

    @property
    def num_tokens(self) -> int:
        return len(self.decode) + sum(n for _, n in self.prefill)

    @property
    def empty(self) -> bool:
        return not self.decode and not self.prefill


class Scheduler:
    def __init__(self, allocator, max_num_seqs: int = 256, max_num_batched_tokens: int = 2048,
                 chunked_prefill: bool = True, max_model_len: int = 32768, preemption: str = "recompute",
                 swap_blocks: int = 0):
        if preemption not in ("recompute", "swap"):
            raise ValueError("preemption must be 'recompute' or 'swap'")
        self.alloc = allocator
        self.bs = allocator.block_size
        self.max_num_seqs = max_num_seqs
        self.max_tokens = max_num_batched_tokens
        self.chunked = chunked_prefill
        self.max_model_len = max_model_len
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []
        self.free_slots = list(range(max_num_seqs - 1, -1, -1))
        self.num_preemptions = 0
        self.preemption = preemption
        self.swap_capacity = swap_blocks if preemption == "swap" else 0
        self.swap_used = 0
        self.swapped: deque[Sequence] = deque()
        self._allow_preempt = True
        self.blocked = False
        self.num_swap_out = 0
        self.num_swap_in = 0

    def add(self, seq: Sequence) -> None:
        if seq.length > self.max_model_len:
            raise ValueError(f"sequence of {seq.length} tokens exceeds max_model_len {self.max_model_len}")
        self.waiting.append(seq)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.swapped)

    # -------------------------------------------------------------- helpers
    def _blocks_needed(self, seq: Sequence, upto: int) -> int:
        need = (upto + self.bs - 1) // self.bs
        return max(0, need - len(seq.block_ids))

    def _grow(self, seq: Sequence, upto: int) -> bool:
        n = self._blocks_needed(seq, upto)
        if n == 0:
            return True
        try:
            seq.block_ids.extend(self.alloc.allocate(n))
            return True
        except OutOfBlocks:
            return False

    def _release(self, seq: Sequence) -> None:
        if seq.block_ids:
            self.alloc.free(seq.block_ids)
        seq.block_ids = []
        if seq.slot >= 0:
            self.free_slots.append(seq.slot)
            seq.slot = -1

    def _computed_blocks(self, seq: Sequence) -> int:
        return (seq.num_computed + self.bs - 1) // self.bs

    def _preempt_one(self, protect: Sequence, scheduled: set, out: ScheduledBatch) -> bool:
        if not self._allow_preempt:
            return False
        victims = [s for s in self.running if s is not protect and id(s) not in scheduled]
        if not victims:
            return False
        victim = min(victims, key=lambda s: (s.params.priority, -s.arrival))
        self.running.remove(victim)
        out.preempted.append(victim)
        out.preempted_slots.append(victim.slot)
        self.num_preemptions += 1
        nkeep = self._computed_blocks(victim)
        if 0 < nkeep and self.swap_used + nkeep <= self.swap_capacity:
            out.swap_out.append((victim, list(victim.block_ids[:nkeep])))
            self._release(victim)
            self.swap_used += nkeep
            victim.status = SequenceStatus.SWAPPED
            self.swapped.append(victim)
            self.num_swap_out += 1
            return True
        self._release(victim)
        victim.num_computed = 0
        victim.num_cached_prefix = 0
        victim.status = SequenceStatus.WAITING
        self.waiting.appendleft(victim)
        return True

    def _swap_in(self, out: ScheduledBatch, fresh: set) -> None:
        while self.swapped and len(self.running) < self.max_num_seqs:
            seq = self.swapped[0]
            n = self._computed_blocks(seq)
            if self.alloc.num_free() < n + len(self.running):
                break  # keep a block of headroom per running sequence
            blocks = self.alloc.allocate(n)
            self.swapped.popleft()
            self.swap_used -= n
            seq.block_ids = list(blocks)
            seq.status = SequenceStatus.RUNNING
            seq.slot = self.free_slots.pop()
            self.running.append(seq)
            out.swap_in.append((seq, list(blocks)))
            out.admitted.append(seq)
            fresh.add(id(seq))
            self.num_swap_in += 1

    # ------------------------------------------------------------- schedule
    def schedule(self, allow_preempt: bool = True) -> ScheduledBatch:
        """Build the next step.  ``allow_preempt=False`` (a step is still in flight,
        so running sequences may hold tokens the host has not seen): a sequence
        that cannot grow is skipped for this step instead of preempting another."""
        self._allow_preempt = allow_preempt
        self.blocked = False  # a running sequence could not grow and preemption was not allowed
        out = ScheduledBatch()
        budget = self.max_tokens
        scheduled: set = set()
        # 0) swapped sequences come back first (protected from preemption this step)
        fresh: set = set()
        if self.swapped:
            self._swap_in(out, fresh)
        # 1) running sequences: decodes and unfinished prompt chunks, in arrival order
        for seq in list(self.running):
            if out.preempted and any(seq is v for v in out.preempted):
                continue  # preempted while making room for an earlier one
            if budget <= 0:
                break
            if seq.pending_finish:
                continue  # its last token is in flight; it finishes when the token lands
            if not seq.in_prefill:
                ok = True
                while not self._grow(seq, seq.length):
                    if not self._preempt_one(seq, scheduled | fresh, out):
                        ok = False
                        break
                if not ok:
                    if not scheduled and allow_preempt:
                        raise OutOfBlocks("KV pool too small for a single sequence")
                    self.blocked = not allow_preempt
                    continue
                out.decode.append(seq)
                scheduled.add(id(seq))
                budget -= 1
            else:
                n = min(seq.num_uncomputed, budget) if self.chunked else seq.num_uncomputed
                if n > budget:
                    continue
                ok = True
                while not self._grow(seq, seq.num_computed + n):
                    if not self._preempt_one(seq, scheduled | fresh, out):
                        ok = False
                        break
                if not ok:
                    if not scheduled and allow_preempt:
                        raise OutOfBlocks("KV pool too small for a single sequence")
                    self.blocked = not allow_preempt
                    continue
                out.prefill.append((seq, n))
                scheduled.add(id(seq))
                budget -= n
        # 2) admit waiting sequences (not while swapped ones wait for room: no starvation)
        while self.waiting and not self.swapped and budget > 0 and len(self.running) < self.max_num_seqs:
            seq = self.waiting[0]
            if seq.num_computed == 0 and not seq.block_ids:
                cached = self.alloc.match_prefix(seq.all_ids)
                seq.block_ids = list(cached)
                seq.num_computed = len(cached) * self.bs
                seq.num_cached_prefix = seq.num_computed
            n = seq.num_uncomputed
            if self.chunked:
                n = min(n, budget)
            elif n > budget:
                break
            if not self._grow(seq, seq.num_computed + n):
                break  # pool full: wait for running sequences to finish
            self.waiting.popleft()
            seq.status = SequenceStatus.RUNNING
            seq.slot = self.free_slots.pop()
            self.running.append(seq)
            out.prefill.append((seq, n))
            out.admitted.append(seq)
            budget -= n
        return out

    def finish(self, seq: Sequence, status: SequenceStatus, keep_blocks: bool = False) -> None:
        """Retire ``seq``; computed full blocks stay in the prefix cache."""
        seq.status = status
        if seq in self.running:
            self.running.remove(seq)
        elif seq in self.waiting:
            self.waiting.remove(seq)
        elif seq in self.swapped:
            self.swapped.remove(seq)
            self.swap_used -= self._computed_blocks(seq)
        if seq.block_ids and seq.num_computed > 0:
            self.alloc.commit_prefix(seq.all_ids[:seq.num_computed], seq.block_ids, int(seq.params.priority))
        if not keep_blocks:
            self._release(seq)

    def rollback(self, seq: Sequence, length: int) -> None:
        """Truncate ``seq`` to its first ``length`` tokens (prompt, then output).
        KV of positions below ``length - 1`` stays; the last kept token is
        recomputed by the next step, which also samples the next token.  Pages
        past the new length go back to the allocator; a swapped sequence drops
        its host copy and is recomputed (reference kv_cache.rs:1156-1203)."""
        if length >= seq.length or length < 1:
            return
        npr = len(seq.prompt_ids)
        if length <= npr:
            seq.prompt_ids = seq.prompt_ids[:length]
            seq.output_ids = []
        else:
            seq.output_ids = seq.output_ids[:length - npr]
        if seq in self.swapped:
            self.swapped.remove(seq)
            self.swap_used -= self._computed_blocks(seq)
            seq.num_computed = 0
            seq.status = SequenceStatus.WAITING
            self.waiting.appendleft(seq)
            return
        seq.num_computed = min(seq.num_computed, length - 1)
        keep = (length + self.bs - 1) // self.bs
        if len(seq.block_ids) > keep:
            self.alloc.free(seq.block_ids[keep:])
            seq.block_ids = seq.block_ids[:keep]

    def abort(self, request_id: str) -> list[Sequence]:
        hit = [s for s in list(self.running) + list(self.waiting) + list(self.swapped) if s.request_id == request_id]
        for s in hit:
            self.finish(s, SequenceStatus.FINISHED_ABORTED)
        return hit
