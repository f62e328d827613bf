"""Continuous-batching scheduler with chunked prefill over the GPU block pool.

The reference ``LLMScheduler`` (crates/kapsl-llm/src/scheduler.rs:69-297)
admits a waiting request only if its *whole* prompt fits the token budget and
then runs every running group each step.  This scheduler keeps the same queue
structure (waiting / running, priority-ordered preemption, session groups keep
their blocks) and adds chunked prefill: each step has a budget of
``max_num_batched_tokens``; running decodes take one token each, then prompt
chunks fill the rest, so long prompts never stall decoding.

Preemption frees a victim's blocks and re-queues it for recomputation (the
victim is the lowest-priority, latest-arrived running sequence).
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
    admitted: list = field(default_factory=list)  # moved from waiting to running this step

    @property
    def num_tokens(self) -> int:
        return len(self.decode) + sum(n for _, n in self.prefill)

    @property
    def empty(self) -> bool:
        return not self.decode and not self.prefill


class Scheduler:
    def __init__(self, allocator, max_num_seqs: int = 256, max_num_batched_tokens: int = 2048,
                 chunked_prefill: bool = True, max_model_len: int = 32768):
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

    def add(self, seq: Sequence) -> None:
        if seq.length > self.max_model_len:
            raise ValueError(f"sequence of {seq.length} tokens exceeds max_model_len {self.max_model_len}")
        self.waiting.append(seq)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

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

    def _preempt_one(self, protect: Sequence, scheduled: set) -> bool:
        victims = [s for s in self.running if s is not protect and id(s) not in scheduled]
        if not victims:
            return False
        victim = min(victims, key=lambda s: (s.params.priority, -s.arrival))
        self.running.remove(victim)
        self._release(victim)
        victim.num_computed = 0
        victim.num_cached_prefix = 0
        victim.status = SequenceStatus.WAITING
        self.waiting.appendleft(victim)
        self.num_preemptions += 1
        return True

    # ------------------------------------------------------------- schedule
    def schedule(self) -> ScheduledBatch:
        out = ScheduledBatch()
        budget = self.max_tokens
        scheduled: set = set()
        # 1) running sequences: decodes and unfinished prompt chunks, in arrival order
        for seq in list(self.running):
            if seq not in self.running:  # preempted while making room for an earlier one
                continue
            if budget <= 0:
                break
            if not seq.in_prefill:
                ok = True
                while not self._grow(seq, seq.length):
                    if not self._preempt_one(seq, scheduled):
                        ok = False
                        break
                    out.preempted.append(self.waiting[0])
                if not ok:
                    if not scheduled:
                        raise OutOfBlocks("KV pool too small for a single sequence")
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
                    if not self._preempt_one(seq, scheduled):
                        ok = False
                        break
                    out.preempted.append(self.waiting[0])
                if not ok:
                    if not scheduled:
                        raise OutOfBlocks("KV pool too small for a single sequence")
                    continue
                out.prefill.append((seq, n))
                scheduled.add(id(seq))
                budget -= n
        # 2) admit waiting sequences
        while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
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
        if seq.block_ids and seq.num_computed > 0:
            self.alloc.commit_prefix(seq.all_ids[:seq.num_computed], seq.block_ids)
        if not keep_blocks:
            self._release(seq)

    def abort(self, request_id: str) -> list[Sequence]:
        hit = [s for s in list(self.running) + list(self.waiting) if s.request_id == request_id]
        for s in hit:
            self.finish(s, SequenceStatus.FINISHED_ABORTED)
        return hit
