"""Tensor parallelism over NVLink 5 / NVSwitch.

Layout (Megatron style): QKV and gate/up are column-parallel (each rank holds
its heads / FFN slice), o_proj and down_proj are row-parallel (each rank holds
the matching input slice and produces a partial sum).  The embedding is
replicated and every rank ends each layer with the same residual stream.  The
lm_head is vocabulary-parallel: each rank multiplies its slice of the
vocabulary, selects that slice's top-k candidates, and the candidates (not
the logits) are exchanged (:meth:`TPComm.vocab_sample`); every rank then
draws the same token with the same per-sequence RNG state, so the ranks stay
in lock step without broadcasting tokens.

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
    # candidates per row in the vocabulary-parallel sampler's exchange buffers
    SAMPLE_K = 1024

    def __init__(self, world_size: int, rank: int, device, mode: str = "fused", group=None,
                 max_tokens: int = 4096, hidden: int = 4096, ep_rows: int = 0, timeout_s: float = 5.0):
        """``timeout_s`` bounds every device-side wait on a peer (flag barriers of the
        fused reduction, the MoE combine and the sampler's candidate exchange): a
        wait that runs out records an error code (see ``ops.check_errors``) and
        the kernel returns instead of hanging."""
        import torch.distributed as dist

        assert mode in ("fused", "scatter", "nccl")
        self.timeout_ns = int(timeout_s * 1e9)
        self.sample_rows = 0
        self.cand_local = None
        self.dist = dist
        self.world_size = world_size
        self.rank = rank
        self.device = torch.device(device)
        self.mode = mode
        self.group = group
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.ep_rows = ep_rows
        # Row counts up to which the fused layer boundary uses the flag-carrying-line
        # kernels: one-shot (every rank reduces every row: one one-way NVLink latency,
        # 2 x (W-1) x rows of traffic), then two-shot (owned rows + all-gather of the
        # normed rows: two one-way latencies, ~4 x rows of traffic); above both, the
        # barrier + pull kernel (half the bytes of two-shot lines, two flag barriers).
        self.ll1_rows = int(os.environ.get("KAPSL_TP_LL1_ROWS", {2: 64, 4: 32, 8: 16}.get(world_size, 0)))
        self.ll2_rows = int(os.environ.get("KAPSL_TP_LL2_ROWS", {2: 512, 4: 512, 8: 512}.get(world_size, 0)))
        # "ll": flag-carrying lines for few rows, pull above (default); "pull": barrier + pull kernel only
        self.norm_kernel = os.environ.get("KAPSL_TP_NORM", "ll")
        # above the line-kernel sizes: "scatter" (the GEMM epilogue stores each row into its
        # owner's receive slot over NVLink while the GEMM runs; the reduction then reads local
        # memory) or "pull" (the reduction pulls the partial rows from the peers)
        self.large_kernel = os.environ.get("KAPSL_TP_LARGE", "scatter")
        self._sms = torch.cuda.get_device_properties(self.device).multi_processor_count if \
            self.device.type == "cuda" else 148
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

    def configure(self, max_tokens: int, hidden: int, ep_rows: int = 0, sample_rows: int = 0) -> None:
        """(Re)size the symmetric buffers once the model geometry is known.
        ``ep_rows``: rows of the expert-output buffer that peers read in the
        fused MoE combine (0 for dense models); ``sample_rows``: rows the
        vocabulary-parallel sampler exchanges candidates for."""
        if self.world_size > 1 and sample_rows > self.sample_rows:
            self.sample_rows = sample_rows
            self.samp_ctr = torch.zeros(2, dtype=torch.int64, device=self.device)
            if self.mode == "nccl":
                self.cand_local = torch.zeros(2, self.world_size, sample_rows, self.SAMPLE_K, 2, dtype=torch.float32,
                                              device=self.device)
            elif self.bufs is not None:
                self.close()
                self.bufs = None
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
        flag_bytes = 4 * 8 * 8  # sites: 0/1 reduction barriers, 2 sampler candidates, 3 spare
        ep_bytes = self.ep_rows * hidden * 2
        cand_bytes = 2 * W * self.sample_rows * self.SAMPLE_K * 8
        xn_bytes = rows_pad * hidden * 2
        # flag-carrying-line slots (reduce slots, then gather slots): rows of one source per parity
        self.ll_cap = max(min(self.ll1_rows, rows_pad), -(-min(self.ll2_rows, rows_pad) // W), 1)
        ll_bytes = c.tp_ll_slot_bytes(W, self.ll_cap, hidden, True)
        align = lambda n: (n + 255) // 256 * 256
        total = (align(recv_bytes) + align(hid_bytes) + align(flag_bytes) + align(ep_bytes) + align(cand_bytes)
                 + align(xn_bytes) + align(ll_bytes))
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
        off_c = off_e + align(ep_bytes)
        off_x = off_c + align(cand_bytes)
        off_ll = off_x + align(xn_bytes)
        ll_half = ll_bytes // 2
        self.bufs = {
            "base": base, "bases": bases, "rpr": rpr, "rows_pad": rows_pad,
            "recv": [b for b in bases], "hidden": [b + off_h for b in bases], "flags": [b + off_f for b in bases],
            "ep": [b + off_e for b in bases], "cand": [b + off_c for b in bases], "xnorm": [b + off_x for b in bases],
            "ll": [b + off_ll for b in bases], "llg": [b + off_ll + ll_half for b in bases],
        }
        # this rank's own partial for the line kernels (the row-parallel GEMM output; read locally)
        self.own_buf = torch.empty(rows_pad, hidden, dtype=torch.bfloat16, device=self.device)
        self.xnorm_buf = c.tensor_from_ptr(base + off_x, [rows_pad, hidden], "bfloat16", self.device.index)
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

    # ------------------------------------------------------ vocab-parallel sampling
    def vocab_sample(self, logits: torch.Tensor, vocab_start: int, vocab_size: int, temperature, top_k, top_p,
                     rng, out, rep_penalty=None, counts=None, slots=None, occ=None, occ_n=None) -> None:
        """Sample from logits split over the ranks by vocabulary (``logits`` holds
        columns [vocab_start, vocab_start + logits.shape[1]) of every row).  Each
        rank selects its slice's top-k candidates; in fused mode the select
        kernel stores them into every peer's candidate buffer and a merge kernel
        (after a bounded wait on the peers' flags) finishes every row; in NCCL
        mode an all-gather moves them.  All ranks draw the same tokens."""
        c = cuda_ops()
        err = ops.error_buffer(logits.device)
        B = logits.shape[0]
        if B > self.sample_rows:
            raise ValueError(f"{B} sampling rows exceed the sampler exchange buffers ({self.sample_rows})")
        W, r = self.world_size, self.rank
        if self.bufs is not None:
            c.sample(logits, temperature, top_k, top_p, rep_penalty, counts, slots, rng, out, occ, occ_n,
                     int(vocab_start), int(vocab_size), None, 0, list(self.bufs["cand"]), list(self.bufs["flags"]),
                     r, self.sample_rows, self.samp_ctr, self.timeout_ns, err)
            return
        local = self.cand_local.data_ptr()
        ptrs = [0] * W
        ptrs[r] = local
        c.sample(logits, temperature, top_k, top_p, rep_penalty, counts, slots, rng, out, occ, occ_n,
                 int(vocab_start), int(vocab_size), None, 0, ptrs, [], r, self.sample_rows, self.samp_ctr, 0, err)
        blk = self.cand_local[0]
        self.dist.all_gather_into_tensor(blk.view(-1), blk[r].reshape(-1), group=self.group)
        c.sample_merge(logits, temperature, top_k, top_p, slots, rng, out, int(vocab_size), [local] * W, r,
                       self.sample_rows, self.samp_ctr, err)

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

    @property
    def fused_norm(self) -> bool:
        """The fused pull reduction can also apply the next RMSNorm (sharded residual)."""
        return self.bufs is not None and self.mode == "fused" and self.world_size in (2, 4, 8)

    def norm_input(self, T: int) -> torch.Tensor:
        """The symmetric buffer the fused reduction writes the next GEMM's input into."""
        return self.xnorm_buf[:T]

    def row_parallel_norm(self, x: torch.Tensor, w, h: torch.Tensor, norm_w: torch.Tensor,
                          eps: float) -> torch.Tensor:
        """``h += all_reduce(x @ w.T)`` then returns ``rmsnorm(h) * norm_w`` for every
        row: one GEMM into a local partial buffer, then one kernel chosen by the
        row count T.  T <= ll1_rows: one-shot flag-carrying lines (every rank
        reduces every row, h stays replicated); T <= ll2_rows: two-shot lines
        (the owner of a row reduces it, h is sharded by rows, the normed rows are
        pushed to every rank); larger T: flag barrier, pull of the owned rows'
        partials from every peer, residual add, RMSNorm, P2P stores of the
        normed rows, barrier.  Every variant sums h + partial_0 + ... +
        partial_{W-1} in rank order, so they agree bit for bit."""
        T = x.shape[0]
        b = self.bufs
        rpr = (T + self.world_size - 1) // self.world_size
        err = ops.error_buffer(x.device)
        if self.norm_kernel == "pull":
            ops.linear(x, w, out=self.partial_buf[:T])
            cuda_ops().tp_reduce_norm_ag(b["recv"], b["xnorm"], b["flags"], h, norm_w, float(eps), self.rank, rpr, T,
                                         self.hidden, self.epoch, err, self.timeout_ns)
            return self.xnorm_buf[:T]
        own = self.own_buf[:T]
        if self.norm_kernel == "ll":
            ll1 = T <= min(self.ll1_rows, self.ll_cap)
            if ll1 or (T <= self.ll2_rows and rpr <= self.ll_cap):
                if isinstance(w, torch.Tensor):  # split-K partials are summed inside the line kernel
                    ws = ops.workspace(x.device)
                    splits = cuda_ops().gemm_deferred(x, w, own, ws, err)
                else:
                    ws, splits = None, 1
                    ops.linear(x, w, out=own)
                cuda_ops().tp_ll_norm(own, b["ll"], b["llg"], h, self.xnorm_buf[:T], norm_w, float(eps), self.rank,
                                      rpr, T, self.ll_cap, not ll1, self.epoch, err, self.timeout_ns, ws, int(splits))
                return self.xnorm_buf[:T]
            if self._scatter_ok(x, w):
                # the epilogue pushed every row into its owner's slot [my rank]; the reduction
                # reads slot p of this rank where the pull variant would read peer p's partial
                cuda_ops().gemm_scatter(x, w, b["recv"], self.rank, rpr, self.hidden, err)
                my, r0, row_bytes = b["recv"][self.rank], self.rank * rpr, self.hidden * 2
                parts = [my + (p * rpr - r0) * row_bytes for p in range(self.world_size)]
            else:
                ops.linear(x, w, out=self.partial_buf[:T])
                parts = b["recv"]
            cuda_ops().tp_reduce_norm_ag(parts, b["xnorm"], b["flags"], h, norm_w, float(eps), self.rank, rpr, T,
                                         self.hidden, self.epoch, err, self.timeout_ns)
            return self.xnorm_buf[:T]
        raise ValueError(f"unknown tensor-parallel norm kernel {self.norm_kernel!r}")

    def _scatter_ok(self, x: torch.Tensor, w) -> bool:
        """The scatter GEMM runs its coalesced epilogue in the 2-SM kernel, chosen when
        256 x 256 tiles fill at least 3/4 of the CTA pairs (the GEMM's own rule)."""
        if self.large_kernel != "scatter" or not isinstance(w, torch.Tensor) or self.hidden % 8:
            return False
        T, N = x.shape[0], w.shape[0]
        units = -(-T // 256) * -(-N // 256)
        return T >= 256 and units * 4 >= (self._sms // 2) * 3

    def replicated_residual(self, T: int) -> bool:
        """Whether the fused row reduction of a ``T``-row batch keeps every row of the
        residual stream current on every rank (one-shot) or only the owned rows."""
        return self.norm_kernel == "ll" and T <= min(self.ll1_rows, self.ll_cap)

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
                           self.epoch, err, self.timeout_ns)
        else:
            ops.linear(x, w, out=self.partial_buf[:T])
            c.tp_pull_reduce_ag(b["recv"], b["hidden"], b["flags"], self.rank, rpr, T, self.hidden, self.hidden,
                                self.epoch, err, self.timeout_ns)
