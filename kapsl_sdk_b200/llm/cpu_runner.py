"""Model runner for the CPU backend: same contract as
:class:`~kapsl_sdk_b200.llm.model_runner.ModelRunner` (``admit``,
``execute``, ``launch`` / ``collect``, ``logits``) with host-side sampling
that reproduces the reference sampler bit for bit (per-sequence LCG state
kept on the sequence).  ``launch`` computes the step at once; ``collect``
hands its tokens over.  A decode input token that the engine has not applied
yet (``Sequence.pending``) is taken from the previous launch's tokens."""
from __future__ import annotations

import time

import numpy as np
import torch

from ..ops import reference as ref
from .scheduler import ScheduledBatch


class CPUModelRunner:
    def __init__(self, model, pool):
        self.model = model
        self.pool = pool
        self.bs = pool.layout.block_size
        self.launches = 0
        self.last_prepare_s = 0.0
        self.stats = {"steps": 0, "graph_steps": 0, "h2d_bytes": 0, "d2h_bytes": 0}
        self.prof = None
        self._step_id = 0
        self._prev = (0, np.zeros(0, dtype=np.int64))  # (step id, tokens) of the last launch

    def launch(self, batch: ScheduledBatch):
        from .model_runner import Inflight

        sid, toks = self._prev
        for s in batch.decode:  # its last output token is the previous launch's sample
            if s.pending is not None:
                if s.pending[0] != sid:
                    raise RuntimeError("pending token from a step other than the previous one")
                s.output_ids[-1] = int(toks[s.pending[1]])
        seqs, toks = self.execute(batch)
        self._step_id += 1
        self._prev = (self._step_id, toks)
        return Inflight(self._step_id, seqs, len(seqs), toks, None, None, "cpu", batch.num_tokens)

    def collect(self, inf):
        return inf.seqs, np.asarray(inf.h_out).copy()

    def admit(self, seqs: list) -> None:
        return None

    def reset_slots(self, seqs: list) -> None:
        return None  # sampler state and penalty counts live on the host sequences

    def _prepare(self, batch: ScheduledBatch):
        ids, pos, slots, seqs, rows, sample = [], [], [], [], [], []
        t = 0
        for s in batch.decode:
            p = s.length - 1
            ids.append(s.output_ids[-1] if s.output_ids else s.prompt_ids[-1])
            pos.append(p)
            slots.append(s.block_ids[p // self.bs] * self.bs + p % self.bs)
            seqs.append((t, 1, s.length, s.block_ids))
            rows.append(t)
            sample.append(s)
            t += 1
        for s, n in batch.prefill:
            p0 = s.num_computed
            allt = s.prompt_ids + s.output_ids
            for p in range(p0, p0 + n):
                ids.append(allt[p])
                pos.append(p)
                slots.append(s.block_ids[p // self.bs] * self.bs + p % self.bs)
            seqs.append((t, n, p0 + n, s.block_ids))
            if p0 + n >= s.length:
                rows.append(t + n - 1)
                sample.append(s)
            t += n
        return (torch.tensor(ids), torch.tensor(pos), torch.tensor(slots), seqs, rows, sample)

    def logits(self, batch: ScheduledBatch) -> torch.Tensor:
        ids, pos, slots, seqs, rows, _ = self._prepare(batch)
        with torch.no_grad():
            return self.model.forward(ids, pos, slots, seqs, self.pool.k, self.pool.v, rows)

    def execute(self, batch: ScheduledBatch):
        t0 = time.perf_counter()
        ids, pos, slots, seqs, rows, sample = self._prepare(batch)
        self.last_prepare_s = time.perf_counter() - t0
        with torch.no_grad():
            out = self.model.forward(ids, pos, slots, seqs, self.pool.k, self.pool.v, rows)
        toks = np.zeros(len(sample), dtype=np.int64)
        if out is None:  # an earlier pipeline stage: the last stage samples and broadcasts
            self.stats["steps"] += 1
            return sample, toks
        lg = out.numpy()
        for r, s in enumerate(sample):
            p = s.params
            row = lg[r]
            if p.repetition_penalty != 1.0:
                row = ref.apply_repetition_penalty(row, s.prompt_ids + s.output_ids, p.repetition_penalty)
            tok, s.rng_state = ref.sample_next_token(row, p.temperature, p.top_k, p.top_p, s.rng_state)
            toks[r] = tok
        self.stats["steps"] += 1
        return sample, toks

    def release_graphs(self) -> None:
        return None
