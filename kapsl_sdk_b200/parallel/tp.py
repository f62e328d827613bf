"""Tensor parallelism over NVLink 5 / NVSwitch.

Layout (Megatron style): QKV and gate/up are column-parallel (each rank holds
its heads / FFN slice), o_proj and down_proj are row-parallel (each rank holds
the matching input slice and produces a partial sum).  The embedding and
lm_head are replicated, so every rank ends each layer with the same residual
stream, computes the same logits and samples the same token with the same
per-sequence RNG state: the ranks stay in lock step without gathering logits
or broadcasting tokens.

Two reduction modes for the row-parallel layers:

* ``"fused"`` (default): each rank's GEMM writes its partial sums into its own
  symmetric buffer (memory every peer maps with CUDA IPC); ``tp_pull_reduce_ag``
  then, after a bounded flag barrier, loads the rows this rank owns from every
  peer's partial buffer over NVLink, adds them and the residual, and stores the
  reduced rows into every rank's residual stream (the all-gather), followed by
  a second barrier.  NVLink traffic of one reduce-scatter plus one all-gather.
* ``"scatter"``: the GEMM epilogue itself stores every partial row into the
  receive slot of the rank that owns it (``gemm_scatter``), and
  ``tp_reduce_ag`` sums the slots locally — the push variant of the same
  reduction.
* ``"nccl"``: plain GEMM, ``torch.distributed.all_reduce`` (NCCL, NVLS when
  NCCL picks it), residual add — the baseline.

Reference counterpart: ``MeshComm`` / ``NcclComm`` (crates/kapsl-hal/src/
device_mesh.rs:427-500, nccl_comm.rs), which stage every collective through
host memory and are not used by any model path.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from .. import ops
from .._ext import cuda_ops


class TPComm:
    def __init__(self, world_size: int, rank: int, device, mode: str = "fused", group=None,
                 max_tokens: int = 4096, hidden: int = 4096, ep_rows: int = 0):
        import torch.distributed as dist

        assert mode in ("fused", "scatter", "nccl")
        self.dist = dist
        self.world_size = world_size
        self.rank = rank
        self.device = torch.device(device)
        self.mode = mode
        self.group = group
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.ep_rows = ep_rows
        self.bufs = None
        self.ep_buf = None
        if mode != "nccl" and world_size > 1:
            self._setup_symmetric(max_tokens, hidden)

    @classmethod
    def from_world(cls, mode: Optional[str] = None, max_tokens: int = 4096, hidden: int = 4096) -> "TPComm":
        import torch.distributed as dist

        mode = mode or os.environ.get("KAPSL_TP_MODE", "fused")
        return cls(dist.get_world_size(), dist.get_rank(), torch.device("cuda", torch.cuda.current_device()), mode,
                   max_tokens=max_tokens, hidden=hidden)

    def configure(self, max_tokens: int, hidden: int, ep_rows: int = 0) -> None:
        """(Re)size the symmetric buffers once the model geometry is known.
        ``ep_rows``: rows of the expert-output buffer that peers read in the
        fused MoE combine (0 for dense models)."""
        if self.mode != "nccl" and self.world_size > 1 and (max_tokens > self.max_tokens or hidden != self.hidden
                                                              or ep_rows > self.ep_rows or self.bufs is None):
            self.close()
            self.max_tokens, self.hidden, self.ep_rows = max_tokens, hidden, max(ep_rows, self.ep_rows)
            self._setup_symmetric(max_tokens, hidden)

    # ------------------------------------------------------- symmetric memory
    def _setup_symmetric(self, max_tokens: int, hidden: int) -> None:
        c = cuda_ops()
        W = self.world_size
        rpr = (max_tokens + W - 1) // W
        rows_pad = rpr * W
        recv_bytes = W * rpr * hidden * 2
        hid_bytes = rows_pad * hidden * 2
        flag_bytes = 2 * 8 * 8
        ep_bytes = self.ep_rows * hidden * 2
        align = lambda n: (n + 255) // 256 * 256
        total = align(recv_bytes) + align(hid_bytes) + align(flag_bytes) + align(ep_bytes)
        base = c.symm_alloc(total)
        handle = c.symm_handle(base)
        handles = [None] * W
        self.dist.all_gather_object(handles, handle, group=self.group)
        bases = []
        for p in range(W):
            bases.append(base if p == self.rank else c.symm_open(handles[p]))
        off_h = align(recv_bytes)
        off_f = off_h + align(hid_bytes)
        off_e = off_f + align(flag_bytes)
        self.bufs = {
            "base": base, "bases": bases, "rpr": rpr, "rows_pad": rows_pad,
            "recv": [b for b in bases], "hidden": [b + off_h for b in bases], "flags": [b + off_f for b in bases],
            "ep": [b + off_e for b in bases],
        }
        dev = self.device.index
        self.ep_buf = (c.tensor_from_ptr(base + off_e, [self.ep_rows, hidden], "bfloat16", dev)
                       if self.ep_rows else None)
        self.hidden_buf = c.tensor_from_ptr(base + off_h, [rows_pad, hidden], "bfloat16", dev)
        self.partial_buf = c.tensor_from_ptr(base, [rows_pad, hidden], "bfloat16", dev)  # pull mode: own partial
        # [0] barrier epoch, [1] finished-CTA count, [2..5] %globaltimer phase stamps of the last
        # call, [8..11] running sums (ns) of the barrier-1 wait, the data phase, the barrier-2
        # wait, and the number of calls of the pull reduction (see :meth:`phase_times`)
        self.epoch = torch.zeros(16, dtype=torch.int64, device=self.device)
        torch.cuda.synchronize(self.device)
        self.dist.barrier(group=self.group)

    def close(self) -> None:
        if self.bufs is None:
            return
        c = cuda_ops()
        torch.cuda.synchronize(self.device)
        self.dist.barrier(group=self.group)
        for p, b in enumerate(self.bufs["bases"]):
            if p != self.rank:
                c.symm_close(b)
        c.symm_free(self.bufs["base"])
        self.bufs = None

    def phase_times(self, reset: bool = False) -> dict:
        """Accumulated device-side phase times of the fused pull reduction
        (read from the kernel's %globaltimer stamps): mean microseconds per
        call of the first barrier, the data phase and the second barrier."""
        if self.bufs is None:
            return {}
        v = self.epoch[8:12].tolist()
        n = max(int(v[3]), 1)
        out = {"calls": int(v[3]), "barrier1_us": v[0] / n / 1e3, "data_us": v[1] / n / 1e3,
               "barrier2_us": v[2] / n / 1e3}
        if reset:
            self.epoch[8:12].zero_()
        return out

    # -------------------------------------------------------------- helpers
    def min_int(self, v: int) -> int:
        t = torch.tensor([int(v)], dtype=torch.int64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN, group=self.group)
        return int(t.item())

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        self.dist.all_reduce(x, group=self.group)
        return x

    def residual_stream(self, T: int) -> Optional[torch.Tensor]:
        """The symmetric residual stream rows [T, hidden] (fused mode), else None."""
        if self.bufs is None:
            return None
        if T > self.bufs["rows_pad"]:
            raise ValueError(f"{T} tokens exceed the tensor-parallel buffers ({self.bufs['rows_pad']})")
        return self.hidden_buf[:T]

    def row_parallel_linear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """NCCL baseline: partial GEMM then all-reduce."""
        y = ops.linear(x, w)
        self.dist.all_reduce(y, group=self.group)
        return y

    def row_parallel_residual(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor) -> None:
        """h += all_reduce(x @ w.T) over the TP group; h is the residual stream."""
        T = x.shape[0]
        if self.bufs is None:
            y = ops.linear(x, w)
            self.dist.all_reduce(y, group=self.group)
            h.add_(y)
            return
        b = self.bufs
        W = self.world_size
        rpr = (T + W - 1) // W
        c = cuda_ops()
        err = ops.error_buffer(x.device)
        if self.mode == "scatter" and isinstance(w, torch.Tensor):  # quantized weights take the pull path
            c.gemm_scatter(x, w, b["recv"], self.rank, rpr, self.hidden, err)
            c.tp_reduce_ag(b["recv"], b["hidden"], b["flags"], self.rank, rpr, T, self.hidden, self.hidden,
                           self.epoch, err)
        else:
            ops.linear(x, w, out=self.partial_buf[:T])
            c.tp_pull_reduce_ag(b["recv"], b["hidden"], b["flags"], self.rank, rpr, T, self.hidden, self.hidden,
                                self.epoch, err)
