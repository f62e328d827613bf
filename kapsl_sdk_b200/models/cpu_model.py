"""fp32 CPU decoder over a paged KV pool (the CPU backend).

Serves small models (the tiny-Llama GGUF workload) and is the reference for
the GPU path.  The math is the plain statement in :mod:`kapsl_sdk_b200.ops.reference`;
when the native CPU kernels are built (``kapsl_sdk_b200._native``) paged
attention runs in C++ over the block table instead of gathering pages.

Reference counterpart: the CPU kernels ``CpuAttention`` / ``CpuMlp``
(crates/kapsl-kernels/src/attention/mod.rs:8-99, mlp/mod.rs:13-49), which the
reference engine never calls; its CPU execution goes through ONNX Runtime or
llama.cpp instead.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import numpy as np
import torch

from ..ops import reference as ref
from ..quantization import PackedRows, RowStack
from .config import ModelConfig


def _mm(x: torch.Tensor, w) -> torch.Tensor:
    """x @ w.T for an fp32 weight or kept-packed GGUF rows."""
    return x @ w.T if isinstance(w, torch.Tensor) else w.matmul(x)


def _cat_rows(parts: list):
    """Row-concatenation of weights: packed rows of one format stay one packed
    matrix, mixed formats (Q4_K_M's Q4_K q/k with a Q6_K v) a RowStack."""
    if all(isinstance(p, torch.Tensor) for p in parts):
        return torch.cat(parts, 0)
    if all(isinstance(p, PackedRows) for p in parts) and len({type(p) for p in parts}) == 1:
        return type(parts[0]).cat(parts)
    return RowStack(parts)


class CPUCausalLM:
    def __init__(self, cfg: ModelConfig, embed: torch.Tensor, lm_head: torch.Tensor, final_norm: torch.Tensor,
                 layers: list):
        def f(t):
            if t is None or isinstance(t, (PackedRows, RowStack)):
                return t
            return t.detach().to("cpu", torch.float32).contiguous()
        self.cfg = cfg
        self.embed = f(embed)
        self.lm_head = f(lm_head)
        self.final_norm = f(final_norm)
        self.layers = []
        for L in layers:
            d = {k: f(v) for k, v in L.items()}
            d["qkv"] = _cat_rows([d["q"], d["k"], d["v"]])
            d["qkv_b"] = torch.cat([d["q_b"], d["k_b"], d["v_b"]]) if d.get("q_b") is not None else None
            if not cfg.is_moe:
                d["gate_up"] = _cat_rows([d["gate"], d["up"]])
            self.layers.append(d)
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, scaling=cfg.rope_scaling)
        self.hq, self.hkv, self.D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        self.scale = cfg.attn_scale if cfg.attn_scale is not None else 1.0 / math.sqrt(self.D)
        self.device = torch.device("cpu")
        self.stage = None  # PipelineStage when this model holds one pipeline stage's layers
        self._k = None  # C++ CPU kernels (kapsl_sdk_b200._native.cpu) when built
        if os.environ.get("KAPSL_CPU_KERNELS", "native") == "native":
            try:
                from .._ext import native

                self._k = native().cpu
            except Exception:
                self._k = None
        if (cfg.act != "silu" or cfg.embed_scale != 1.0 or cfg.attn_softcap or cfg.final_softcap
                or cfg.sliding_pattern or any("attn_out_norm" in L for L in self.layers)):
            self._k = None  # GeGLU / soft-capping / windows / sandwich norms: the PyTorch statement

    @classmethod
    def random(cls, cfg: ModelConfig, seed: int = 0, std: float = 0.02, layers: Optional[range] = None,
               stage=None) -> "CPUCausalLM":
        """Random weights from ``seed``; with ``layers`` (a pipeline stage's range) only
        those layers are kept, drawn from the same stream as the full model."""
        from .llama import random_full_weights

        items = list(random_full_weights(cfg, torch.device("cpu"), seed, std))
        full = [t for k, t in items[2:]]
        if layers is not None:
            full = [full[i] for i in layers]
        m = cls(cfg, items[0][1], items[1][1], torch.ones(cfg.hidden_size), full)
        m.stage = stage
        return m

    def forward(self, ids: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, seqs: list,
                k_caches: list, v_caches: list, logits_rows: list) -> torch.Tensor:
        """``seqs``: list of (row_start, n_tokens, ctx_len, block_ids) per sequence;
        returns fp32 logits for ``logits_rows``."""
        if self._k is not None:
            return self._forward_native(ids, positions, slots, seqs, k_caches, v_caches, logits_rows)
        cfg = self.cfg
        T = ids.numel()
        D, hq, hkv = self.D, self.hq, self.hkv
        h = self._stage_input(ids)
        bs = k_caches[0].shape[2]
        layer_ids = self.layer_ids
        blk = (slots // bs).long()
        off = (slots % bs).long()
        for li, L in enumerate(self.layers):
            x, _ = ref.rmsnorm(h, L["in_norm"], cfg.rms_eps)
            qkv = _mm(x, L["qkv"])
            if L["qkv_b"] is not None:
                qkv = qkv + L["qkv_b"]
            q, k = qkv[:, :hq * D].view(T, hq, D), qkv[:, hq * D:(hq + hkv) * D].view(T, hkv, D)
            if L.get("q_norm") is not None:  # Qwen3: per-head RMSNorm before RoPE
                q = ref.rmsnorm(q, L["q_norm"], cfg.rms_eps)[0]
                k = ref.rmsnorm(k, L["k_norm"], cfg.rms_eps)[0]
            q = ref.apply_rope(q, positions, self.cos_sin)
            k = ref.apply_rope(k, positions, self.cos_sin)
            v = qkv[:, (hq + hkv) * D:].view(T, hkv, D)
            kc, vc = k_caches[li], v_caches[li]
            kc[blk, :, off] = k.to(kc.dtype)
            vc[blk, :, off] = v.to(vc.dtype)
            attn = torch.empty(T, hq * D)
            win = cfg.layer_window(layer_ids[li])
            for r0, n, ctx, blocks in seqs:
                kk = ref.gather_paged(kc, blocks, ctx).float()
                vv = ref.gather_paged(vc, blocks, ctx).float()
                attn[r0:r0 + n] = ref.attention(q[r0:r0 + n], kk, vv, self.scale, ctx - n, cfg.attn_softcap,
                                                win).reshape(n, hq * D)
            o = _mm(attn, L["o"])
            if "attn_out_norm" in L:  # Gemma 2: norm of the attention output before the residual add
                o, _ = ref.rmsnorm(o, L["attn_out_norm"], cfg.rms_eps)
            h = h + o
            x, _ = ref.rmsnorm(h, L["post_norm"], cfg.rms_eps)
            if cfg.is_moe:
                h = h + self._moe(x, L)
            else:
                gu = _mm(x, L["gate_up"])
                y = _mm(ref.gelu_tanh_mul(gu) if cfg.act == "gelu_tanh" else ref.silu_mul(gu), L["down"])
                if "mlp_out_norm" in L:
                    y, _ = ref.rmsnorm(y, L["mlp_out_norm"], cfg.rms_eps)
                h = h + y
        if self.stage is not None and not self.stage.last:
            self.stage.send_hidden(h)
            return None
        xs, _ = ref.rmsnorm(h[logits_rows], self.final_norm, cfg.rms_eps)
        logits = _mm(xs, self.lm_head)
        if cfg.final_softcap > 0:
            logits = torch.tanh(logits / cfg.final_softcap) * cfg.final_softcap
        return logits

    def _forward_native(self, ids, positions, slots, seqs, k_caches, v_caches, logits_rows) -> torch.Tensor:
        """Same computation with the C++ CPU kernels between the BLAS matmuls."""
        k_ = self._k
        cfg = self.cfg
        T = ids.numel()
        D, hq, hkv = self.D, self.hq, self.hkv
        h = self._stage_input(ids).contiguous()
        pos = positions.to(torch.int64).contiguous().numpy()
        sl = slots.to(torch.int64).contiguous().numpy()
        row0 = np.array([r for r, _, _, _ in seqs], dtype=np.int64)
        nq = np.array([n for _, n, _, _ in seqs], dtype=np.int64)
        ctx = np.array([c for _, _, c, _ in seqs], dtype=np.int64)
        mb = max(len(b) for _, _, _, b in seqs)
        bt = np.zeros((len(seqs), mb), dtype=np.int32)
        for i, (_, _, _, b) in enumerate(seqs):
            bt[i, :len(b)] = b
        cs = self.cos_sin.numpy()
        x = torch.empty_like(h)
        attn = torch.empty(T, hq, D)
        for li, L in enumerate(self.layers):
            k_.rmsnorm(h.numpy(), L["in_norm"].numpy(), x.numpy(), cfg.rms_eps)
            qkv = _mm(x, L["qkv"])
            if L["qkv_b"] is not None:
                qkv += L["qkv_b"]
            q = qkv[:, :hq * D].contiguous().view(T, hq, D)
            kk = qkv[:, hq * D:(hq + hkv) * D].contiguous().view(T, hkv, D)
            vv = qkv[:, (hq + hkv) * D:].contiguous().view(T, hkv, D)
            if L.get("q_norm") is not None:  # Qwen3: per-head RMSNorm before RoPE
                qn, kn = q.view(T * hq, D), kk.view(T * hkv, D)
                k_.rmsnorm(qn.numpy(), L["q_norm"].numpy(), qn.numpy(), cfg.rms_eps)
                k_.rmsnorm(kn.numpy(), L["k_norm"].numpy(), kn.numpy(), cfg.rms_eps)
            k_.rope(q.numpy(), pos, cs)
            k_.rope(kk.numpy(), pos, cs)
            kc, vc = k_caches[li], v_caches[li]
            k_.kv_write(kk.numpy(), vv.numpy(), sl, kc.numpy(), vc.numpy())
            k_.paged_attention(q.numpy(), kc.numpy(), vc.numpy(), row0, nq, ctx, bt, self.scale, attn.numpy())
            h += _mm(attn.view(T, hq * D), L["o"])
            k_.rmsnorm(h.numpy(), L["post_norm"].numpy(), x.numpy(), cfg.rms_eps)
            if cfg.is_moe:
                h += self._moe(x, L)
            else:
                gu = _mm(x, L["gate_up"])
                act = torch.empty(T, gu.shape[1] // 2)
                k_.silu_mul(gu.numpy(), act.numpy())
                h += _mm(act, L["down"])
        if self.stage is not None and not self.stage.last:
            self.stage.send_hidden(h)
            return None
        xs = h[logits_rows].contiguous()
        k_.rmsnorm(xs.numpy(), self.final_norm.numpy(), xs.numpy(), cfg.rms_eps)
        return _mm(xs, self.lm_head)

    @property
    def layer_ids(self) -> list:
        """Global index of each held layer (a pipeline stage holds a contiguous range)."""
        return list(self.stage.layers) if self.stage is not None else list(range(len(self.layers)))

    def _stage_input(self, ids: torch.Tensor) -> torch.Tensor:
        """Token embeddings, or (later pipeline stages) the previous stage's hidden state."""
        if self.stage is not None and not self.stage.first:
            return self.stage.recv_hidden(ids.numel(), self.cfg.hidden_size, torch.float32, self.device)
        h = self.embed[ids.long()]
        return h * self.cfg.embed_scale if self.cfg.embed_scale != 1.0 else h

    def _moe(self, x: torch.Tensor, L: dict) -> torch.Tensor:
        cfg = self.cfg
        p = torch.softmax(x @ L["router"].T, -1)
        topv, topi = p.topk(cfg.experts_per_token, -1)
        topv = topv / topv.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        for e in range(cfg.num_experts):
            sel = topi == e
            rows = sel.any(-1).nonzero().flatten()
            if rows.numel() == 0:
                continue
            w = (topv * sel).sum(-1)[rows]
            xe = x[rows]
            g = xe @ L["experts_gate"][e].T
            u = xe @ L["experts_up"][e].T
            out[rows] += w[:, None] * ((g * torch.sigmoid(g) * u) @ L["experts_down"][e].T)
        return out
