"""Pipeline parallelism: each rank of the pipeline group owns a contiguous
range of decoder layers.

Per engine step every stage runs the same scheduler (all stages receive the
same requests, so their decisions match), splits the step's sequences into
``micro_batches`` groups and, for each group in order: receives the hidden
state from the previous stage (stage 0 embeds the tokens instead), runs its
layers (writing its own layers' KV pages) and sends the result on with a
non-blocking point-to-point send.  While stage s works on group m, stage s+1
works on group m-1, so the stages overlap.  The last stage applies the final
norm and lm_head and samples; once all groups are done it broadcasts the
step's tokens to every stage, which all append the same tokens.

Transport: ``torch.distributed`` point-to-point (NCCL between GPUs, gloo on
CPU), overlapped with compute by the non-blocking sends.

Reference counterpart: ONNX pipeline stages run one after another per
sequence, with outputs handed over on the host
(crates/kapsl-llm/src/engine.rs:1705-1772, 4869-5460).
"""
from __future__ import annotations

from typing import Optional

import torch


def stage_layers(num_layers: int, num_stages: int, stage: int) -> range:
    """Contiguous, balanced split (earlier stages take the remainder)."""
    base, rem = divmod(num_layers, num_stages)
    start = stage * base + min(stage, rem)
    return range(start, start + base + (1 if stage < rem else 0))


class PipelineStage:
    def __init__(self, stage: int, num_stages: int, num_layers: int, ranks: Optional[list] = None, group=None,
                 micro_batches: int = 2):
        import torch.distributed as dist

        self.dist = dist
        self.stage, self.num_stages = stage, num_stages
        self.layers = stage_layers(num_layers, num_stages, stage)
        self.ranks = ranks or list(range(num_stages))
        self.group = group
        self.micro_batches = max(1, micro_batches)
        self._pending: list = []

    @property
    def first(self) -> bool:
        return self.stage == 0

    @property
    def last(self) -> bool:
        return self.stage == self.num_stages - 1

    def recv_hidden(self, rows: int, width: int, dtype, device) -> torch.Tensor:
        h = torch.empty(rows, width, dtype=dtype, device=device)
        self.dist.recv(h, src=self.ranks[self.stage - 1], group=self.group)
        return h

    def send_hidden(self, h: torch.Tensor) -> None:
        h = h.contiguous()
        self._pending.append((self.dist.isend(h, dst=self.ranks[self.stage + 1], group=self.group), h))

    def wait_sends(self) -> None:
        for w, _ in self._pending:
            w.wait()
        self._pending = []

    def broadcast_tokens(self, toks: torch.Tensor) -> torch.Tensor:
        """The last stage's sampled tokens to every stage (in place)."""
        self.wait_sends()
        self.dist.broadcast(toks, src=self.ranks[-1], group=self.group)
        return toks


def split_batch(batch, parts: int) -> list:
    """Split a ScheduledBatch into up to ``parts`` batches of whole sequences
    (decode rows and prefill chunks spread by token count)."""
    from ..llm.scheduler import ScheduledBatch

    items = [("d", s, 1) for s in batch.decode] + [("p", s, n) for s, n in batch.prefill]
    if parts <= 1 or len(items) <= 1:
        return [batch]
    parts = min(parts, len(items))
    total = sum(n for _, _, n in items)
    out = [ScheduledBatch() for _ in range(parts)]
    i, acc = 0, 0
    for kind, s, n in items:
        if acc >= total * (i + 1) / parts and i < parts - 1 and (out[i].decode or out[i].prefill):
            i += 1
        (out[i].decode.append(s) if kind == "d" else out[i].prefill.append((s, n)))
        acc += n
    admitted = set(id(s) for s in batch.admitted)
    for b in out:
        b.admitted = [s for s in b.decode + [s for s, _ in b.prefill] if id(s) in admitted]
    return [b for b in out if b.decode or b.prefill]
