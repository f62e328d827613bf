"""Kernel traits of the hardware layer: a small, backend-neutral interface to
the attention and MLP kernels, for code that wants them outside the engine.

* :class:`AttentionConfig` — ``scale`` (default 1/sqrt(head_dim)) and
  ``causal`` (query i of Sq sees keys <= Sk - Sq + i).
* :class:`TensorView` — a borrowed (data, shape) view with shape checks.
* :class:`KernelBackend` — ``attention(q, k, v)`` over [B, H, S, D] (GQA when
  k/v have fewer heads), ``paged_attention`` over a block table,
  ``fused_swiglu(g, u)``.  :class:`CpuKernelBackend` runs the C++ CPU kernels
  (fp32), :class:`CudaKernelBackend` the sm_100a kernels (bf16, head_dim 128).
* :func:`create_backend` — picks by device.

Reference: crates/kapsl-hal/src/kernel.rs:6-69 (traits), tensor.rs:3-41
(views) and crates/kapsl-kernels (CPU attention without a block table, and
``create_backend`` that always returns the CPU backend).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch


@dataclass
class AttentionConfig:
    scale: Optional[float] = None
    causal: bool = True

    def scale_for(self, head_dim: int) -> float:
        return self.scale if self.scale is not None else 1.0 / math.sqrt(head_dim)


class TensorView:
    def __init__(self, data, shape: tuple):
        n = int(np.prod(shape)) if shape else 1
        if np.asarray(data).size != n:
            raise ValueError(f"view of {np.asarray(data).size} values cannot have shape {tuple(shape)}")
        self.data, self.shape = data, tuple(shape)

    def as_tensor(self) -> torch.Tensor:
        t = self.data if isinstance(self.data, torch.Tensor) else torch.as_tensor(np.asarray(self.data))
        return t.reshape(self.shape)


class KernelBackend:
    name = "base"

    def attention(self, q, k, v, cfg: Optional[AttentionConfig] = None) -> torch.Tensor:
        raise NotImplementedError

    def paged_attention(self, q, k_cache, v_cache, block_tables, ctx_lens, q_lens, cfg=None) -> torch.Tensor:
        raise NotImplementedError

    def fused_swiglu(self, gate, up) -> torch.Tensor:
        raise NotImplementedError


def _rank4(*ts):
    for t in ts:
        if t.dim() != 4:
            raise ValueError("attention expects [B, H, S, D] tensors")


class CpuKernelBackend(KernelBackend):
    name = "cpu"

    def __init__(self):
        from .._ext import native

        self.k = native().cpu

    def paged_attention(self, q, k_cache, v_cache, block_tables, ctx_lens, q_lens, cfg=None) -> torch.Tensor:
        """q [T, Hq, D] (the sequences' new tokens back to back); caches [blocks, Hkv, bs, D]."""
        cfg = cfg or AttentionConfig()
        q = q.float().contiguous()
        out = torch.empty_like(q)
        row0 = np.concatenate([[0], np.cumsum(np.asarray(q_lens, np.int64))[:-1]]).astype(np.int64)
        self.k.paged_attention(q.numpy(), k_cache.float().contiguous().numpy(), v_cache.float().contiguous().numpy(),
                               row0, np.asarray(q_lens, np.int64), np.asarray(ctx_lens, np.int64),
                               np.ascontiguousarray(np.asarray(block_tables, np.int32)), cfg.scale_for(q.shape[-1]),
                               out.numpy())
        return out

    def attention(self, q, k, v, cfg: Optional[AttentionConfig] = None) -> torch.Tensor:
        cfg = cfg or AttentionConfig()
        _rank4(q, k, v)
        B, Hq, Sq, D = q.shape
        Sk, Hkv = k.shape[2], k.shape[1]
        if not cfg.causal:
            s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float().repeat_interleave(Hq // Hkv, 1))
            p = torch.softmax(s * cfg.scale_for(D), -1)
            return torch.einsum("bhqk,bhkd->bhqd", p, v.float().repeat_interleave(Hq // Hkv, 1))
        # one "page" per sequence holding all its keys, then the paged kernel
        kc = k.float().contiguous()  # [B, Hkv, Sk, D] == [blocks, Hkv, bs=Sk, D]
        vc = v.float().contiguous()
        qq = q.float().permute(0, 2, 1, 3).reshape(B * Sq, Hq, D)
        out = self.paged_attention(qq, kc, vc, [[b] for b in range(B)], [Sk] * B, [Sq] * B, cfg)
        return out.view(B, Sq, Hq, D).permute(0, 2, 1, 3).contiguous()

    def fused_swiglu(self, gate, up) -> torch.Tensor:
        x = torch.cat([gate.float(), up.float()], -1).contiguous()
        flat = x.reshape(-1, x.shape[-1])
        out = torch.empty(flat.shape[0], gate.shape[-1])
        self.k.silu_mul(flat.numpy(), out.numpy())
        return out.view(gate.shape)


class CudaKernelBackend(KernelBackend):
    name = "cuda"

    def paged_attention(self, q, k_cache, v_cache, block_tables, ctx_lens, q_lens, cfg=None) -> torch.Tensor:
        from .. import ops

        cfg = cfg or AttentionConfig()
        T, Hq, D = q.shape
        if D != 128:
            raise ValueError("the sm_100a attention kernels take head_dim 128")
        dev = q.device
        seq_info, t = [], 0
        for s, (n, c) in enumerate(zip(q_lens, ctx_lens)):
            seq_info.append((t, n, c, s))
            t += n
        out = torch.zeros(T, Hq * D, dtype=torch.bfloat16, device=dev)
        ops.prefill_attention(q.to(torch.bfloat16).reshape(T, Hq * D).contiguous(), k_cache.to(torch.bfloat16),
                              v_cache.to(torch.bfloat16),
                              torch.tensor(ops.prefill_work(list(q_lens)), dtype=torch.int32, device=dev),
                              torch.tensor(seq_info, dtype=torch.int32, device=dev),
                              torch.as_tensor(block_tables, dtype=torch.int32, device=dev), Hq, k_cache.shape[1],
                              out, cfg.scale_for(D))
        return out.view(T, Hq, D)

    def fused_swiglu(self, gate, up) -> torch.Tensor:
        from .. import ops

        x = torch.cat([gate, up], -1).to(torch.bfloat16).reshape(-1, 2 * gate.shape[-1]).contiguous()
        return ops.silu_mul(x).view(gate.shape)


def create_backend(device="cpu") -> KernelBackend:
    return CudaKernelBackend() if torch.device(device).type == "cuda" else CpuKernelBackend()
