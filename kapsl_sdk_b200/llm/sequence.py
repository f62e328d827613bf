"""Per-request state for the continuous-batching engine.

Counterpart of crates/kapsl-llm/src/sequence.rs:6-214 (Sequence,
SequenceGroup, SamplingParams).  A request is one sequence here (the reference
``SequenceGroup`` always holds exactly one sequence).
"""
from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field
from typing import Callable, Optional

import numpy as np


@dataclass
class SamplingParams:
    """Defaults follow the reference (crates/kapsl-llm/src/llm_backend.rs:55-65):
    512 new tokens, T=0.7, top_p 0.9, top_k 40, repetition penalty 1.15."""
    max_new_tokens: int = 512
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: int = 40
    repetition_penalty: float = 1.15
    seed: Optional[int] = None
    stop_token_ids: list = field(default_factory=list)
    ignore_eos: bool = False
    priority: int = 0

    @classmethod
    def greedy(cls, max_new_tokens: int = 512, **kw) -> "SamplingParams":
        return cls(max_new_tokens=max_new_tokens, temperature=0.0, top_p=1.0, top_k=0, repetition_penalty=1.0, **kw)


PENDING_TOKEN = -1  # placeholder in output_ids for a token sampled by a step still in flight


class SequenceStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    SWAPPED = "swapped"
    FINISHED_STOPPED = "finished_stopped"
    FINISHED_LENGTH = "finished_length"
    FINISHED_ABORTED = "finished_aborted"

    @property
    def finished(self) -> bool:
        return self.value.startswith("finished")


@dataclass(eq=False)
class Sequence:
    seq_id: int
    request_id: str
    prompt_ids: list
    params: SamplingParams
    rng_state: int = 0
    output_ids: list = field(default_factory=list)
    status: SequenceStatus = SequenceStatus.WAITING
    block_ids: list = field(default_factory=list)
    num_computed: int = 0          # tokens whose KV is in the cache
    num_cached_prefix: int = 0     # tokens reused from the prefix cache at admission
    arrival: float = field(default_factory=time.perf_counter)
    first_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    token_times: list = field(default_factory=list)
    slot: int = -1                 # row in the device penalty-count table
    session_id: Optional[str] = None
    on_token: Optional[Callable] = None
    finish_reason: Optional[str] = None
    # the last output token is still on the device: (step id, sampler row) of the launched
    # step that samples it; output_ids holds PENDING_TOKEN there until the step completes
    pending: Optional[tuple] = None
    pending_finish: bool = False   # the in-flight token is its last (length limit): not scheduled again
    _bt: Optional[tuple] = field(default=None, repr=False)  # (block_ids list, its length, int32 copy)

    def block_table(self) -> np.ndarray:
        """``block_ids`` as an int32 array, rebuilt only when the list was replaced
        or grew (the scheduler only appends to it or assigns a new list)."""
        c, bl = self._bt, self.block_ids
        if c is None or c[0] is not bl or c[1] != len(bl):
            c = (bl, len(bl), np.asarray(bl, dtype=np.int32))
            self._bt = c
        return c[2]

    @property
    def all_ids(self) -> list:
        return self.prompt_ids + self.output_ids

    @property
    def length(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)

    @property
    def num_uncomputed(self) -> int:
        return self.length - self.num_computed

    @property
    def in_prefill(self) -> bool:
        return self.num_computed < len(self.prompt_ids)

    def ttft(self) -> Optional[float]:
        return None if self.first_token_time is None else self.first_token_time - self.arrival

    def tpot(self) -> Optional[float]:
        if self.first_token_time is None or len(self.output_ids) < 2 or self.finish_time is None:
            return None
        return (self.finish_time - self.first_token_time) / (len(self.output_ids) - 1)
