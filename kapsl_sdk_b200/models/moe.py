"""Mixture-of-experts FFN (Mixtral-style top-k routing) with expert parallelism.

Per layer, on every rank::

    ids, w   = moe_route(x)                  # router GEMV + top-k + softmax weights
    seg, pos = moe_permute(ids)              # stable expert sort, 128-row padded segments
    xs       = moe_gather(x)                 # rows bound for this rank's experts
    g        = grouped GEMM (gate/up, SwiGLU epilogue)   tcgen05, device tile table
    y        = grouped GEMM (down)
    h       += combine(w * y[top-k rows])    # fused with the cross-rank reduction

Expert parallelism: experts are split evenly over the ranks of the tensor
parallel group.  The attention block leaves the hidden state replicated on
every rank, so dispatch is a local gather; the combine kernel pulls each token's
k expert rows from the ranks that own them (peer loads over NVLink), adds the
residual and writes the result into every rank's residual stream.  In the NCCL
baseline mode the combine sums the local experts only and an all-reduce adds
the ranks' partial sums.

Reference counterpart: none — the reference has no MoE or expert parallelism
(crates/kapsl-hal/src/device_mesh.rs:5-70 lists only DP/TP/PP topologies).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops
from .config import ModelConfig

BM = 128


def _ceil(a: int, b: int) -> int:
    return (a + b - 1) // b


class MoE:
    def __init__(self, cfg: ModelConfig, device, tp_comm=None, renormalize: bool = True):
        assert cfg.is_moe
        self.cfg = cfg
        self.device = torch.device(device)
        self.tp = tp_comm
        self.world = tp_comm.world_size if tp_comm is not None else 1
        self.rank = tp_comm.rank if tp_comm is not None else 0
        E = cfg.num_experts
        if E % self.world != 0:
            raise ValueError(f"{E} experts cannot be split over {self.world} ranks")
        self.E, self.K = E, cfg.experts_per_token
        self.el = E // self.world
        self.e_lo = self.rank * self.el
        self.renormalize = renormalize
        self.max_tokens = 0
        self.sms = torch.cuda.get_device_properties(self.device).multi_processor_count

    def rows_bound(self, T: int) -> int:
        """Upper bound of the expert-sorted rows this rank can receive for T tokens."""
        return _ceil(T * min(self.K, self.el) + self.el * (BM - 1), BM) * BM

    def configure(self, max_tokens: int) -> None:
        if max_tokens <= self.max_tokens:
            return
        self.max_tokens = max_tokens
        cfg, dev = self.cfg, self.device
        R = self.rows_bound(max_tokens)
        d, F = cfg.hidden_size, cfg.intermediate_size
        i32 = dict(dtype=torch.int32, device=dev)
        self.ids = torch.zeros(max_tokens, self.K, **i32)
        self.wts = torch.zeros(max_tokens, self.K, dtype=torch.float32, device=dev)
        self.seg = torch.zeros(self.E + 1, **i32)
        self.pos = torch.zeros(max_tokens * self.K, **i32)
        self.mtiles = torch.zeros(1 + R // BM, **i32)
        self.src = torch.zeros(R, **i32)
        self.xs = torch.empty(R, d, dtype=torch.bfloat16, device=dev)
        self.g = torch.empty(R, F, dtype=torch.bfloat16, device=dev)
        self.fused = self.world > 1 and self.tp is not None and self.tp.mode != "nccl"
        if self.fused:
            self.tp.configure(max(self.tp.max_tokens, max_tokens), d, ep_rows=R)
            self.y = self.tp.ep_buf
        else:
            self.y = torch.empty(R, d, dtype=torch.bfloat16, device=dev)
            self.partial = torch.empty(max_tokens, d, dtype=torch.bfloat16, device=dev) if self.world > 1 else None

    def _plan(self, T: int, n: int, k: int) -> tuple[int, int]:
        """(tile width, split-K) for a grouped GEMM with n output columns and k inputs."""
        est_mt = self.el * max(1, _ceil(T * self.K, self.E * BM))
        bn = 256 if est_mt * (n // 256) >= self.sms else 128
        units = est_mt * (n // bn)
        splits = 1
        if units < self.sms // 2 and k // 64 >= 8:
            splits = max(1, min(16, self.sms // units, k // 256))  # one wave, every SM streaming
        return bn, splits

    def forward(self, x: torch.Tensor, L, h: torch.Tensor) -> None:
        """h[:T] += MoE(x) (x = post-attention-norm hidden state, [T, d])."""
        T = x.shape[0]
        if T > self.max_tokens:
            self.configure(T)
        cfg = self.cfg
        d, F = cfg.hidden_size, cfg.intermediate_size
        ids, wts = self.ids[:T], self.wts[:T]
        ops.moe_route(x, L.w_router, self.K, self.renormalize, ids, wts)
        R = self.rows_bound(T)
        ops.moe_permute(ids, self.E, self.e_lo, self.el, R, self.seg, self.pos[:T * self.K], self.mtiles, self.src)
        xs, g, y = self.xs[:R], self.g[:R], self.y[:R]
        ops.moe_gather(x, self.src, self.mtiles, xs)
        bn, sp = self._plan(T, 2 * F, d)
        ops.grouped_linear(xs, L.w_experts_gu.view(-1, d), 2 * F, self.mtiles, g, swiglu=True, splits=sp)
        bn, sp = self._plan(T, d, F)
        ops.grouped_linear(g, L.w_experts_down.view(-1, F), d, self.mtiles, y, splits=sp, bn=bn)
        pos = self.pos[:T * self.K]
        if self.world == 1:
            ops.moe_combine([y.data_ptr()], [h.data_ptr()], [], 0, ids, wts, pos, self.seg, self.el, d, y.stride(0),
                            h.stride(0), T)
        elif self.fused:
            b = self.tp.bufs
            rpr = _ceil(T, self.world)
            ops.moe_combine(b["ep"], b["hidden"], b["flags"], self.rank, ids, wts, pos, self.seg, self.el, d, d, d,
                            rpr, self.tp.epoch, self.tp.timeout_ns)
        else:
            part = self.partial[:T]
            part.zero_()
            ops.moe_combine([y.data_ptr()], [part.data_ptr()], [], self.rank, ids, wts, pos, self.seg, self.el, d,
                            y.stride(0), part.stride(0), T)
            self.tp.all_reduce(part)
            h.add_(part)


def reference_moe(x: torch.Tensor, w_router: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                  top_k: int, renormalize: bool = True) -> torch.Tensor:
    """fp32 oracle: x [T, d], gate/up [E, F, d], down [E, d, F] -> [T, d]."""
    x = x.float()
    p = torch.softmax(x @ w_router.float().T, -1)
    topv, topi = p.topk(top_k, -1)
    if renormalize:
        topv = topv / topv.sum(-1, keepdim=True)
    out = torch.zeros_like(x)
    for e in range(w_router.shape[0]):
        sel = topi == e
        rows = sel.any(-1).nonzero().flatten()
        if rows.numel() == 0:
            continue
        wgt = (topv * sel).sum(-1)[rows]
        xe = x[rows]
        gg = xe @ gate[e].float().T
        uu = xe @ up[e].float().T
        out[rows] += wgt[:, None] * ((gg * torch.sigmoid(gg) * uu) @ down[e].float().T)
    return out
