"""The in-repo library baseline ("B1"): the same engine, scheduler, paged KV pool
and CUDA-graph decode as the product, with every model op from a library.

* GEMMs: ``torch.nn.functional.linear`` (cuBLAS), unfused epilogues;
* tensor parallelism: ``torch.distributed.all_reduce`` (NCCL) after the
  row-parallel projections, lm_head replicated on every rank;
* RMSNorm, RoPE, SwiGLU, residual adds: plain PyTorch ops;
* paged KV write and attention: vLLM's ``reshape_and_cache_flash`` and its
  FlashAttention-2 varlen kernel over the block table (16-token pages; the
  pool's [blocks, heads, 16, 128] pages are passed as a strided
  [blocks, 16, heads, 128] view);
* sampling: PyTorch top-k / top-p / multinomial (not the reference's LCG
  stream: this arm measures speed, not seeded reproducibility).

It exists to put a number on "NCCL + cuBLAS + library attention" for the
same workload; the reference itself ships no GPU path to compare with (its
LLM math runs inside ONNX Runtime sessions, crates/kapsl-llm/src/engine.rs:
2885-2890, 3567).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import reference as ref
from .llama import CausalLM, ForwardBatch


def _vllm_ops():
    """vLLM's flash-attention varlen function and cache-write op (library kernels)."""
    import vllm._custom_ops as vops  # noqa: F401  (registers torch.ops._C_cache_ops)
    from vllm.vllm_flash_attn import flash_attn_varlen_func

    return vops, flash_attn_varlen_func


class BaselineCausalLM(CausalLM):
    library_sampler = True

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        if self.moe is not None or self.stage is not None:
            raise ValueError("the library baseline covers dense models without pipeline stages")
        self.vops, self.fa = _vllm_ops()
        self.k_scale = torch.ones(1, dtype=torch.float32, device=self.device)
        self.v_scale = torch.ones(1, dtype=torch.float32, device=self.device)
        self.prefill_tc = False
        self.prefill_tile = 64
        self._arange = torch.arange(4097, dtype=torch.int32, device=self.device)

    def configure_tp(self, max_tokens: int, sample_rows: int = 0) -> None:
        return None  # NCCL only: no symmetric buffers

    def _all_reduce(self, y: torch.Tensor) -> torch.Tensor:
        if self.tp_size > 1:
            self.tp.dist.all_reduce(y, group=self.tp.group)
        return y

    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        return ref.apply_rope(x, pos, self.cos_sin).to(torch.bfloat16)

    def forward(self, fb: ForwardBatch, k_caches: list, v_caches: list, full_vocab: bool = True) -> torch.Tensor:
        cfg = self.cfg
        T, Bd = fb.num_tokens, fb.num_decode
        D, hq, hkv = self.D, self.hq, self.hkv
        ids = fb.input_ids[:T]
        if fb.src_rows is not None:  # decode inputs sampled by the previous step, still on the device
            n = fb.src_rows.numel()
            src = fb.src_rows.long()
            prev = fb.prev_tokens[src.clamp(min=0)]
            ids = torch.cat([torch.where(src >= 0, prev, ids[:n]), ids[n:]])
        h = F.embedding(ids.long(), self.w.embed).float()
        pos = fb.positions[:T]
        # per-sequence metadata for the varlen kernel: decode rows, then the prefill chunks
        S_pf = 0 if fb.pf_seq_info is None else fb.pf_seq_info.shape[0]
        if S_pf:
            pf = fb.pf_seq_info
            qlens = torch.cat([torch.ones(Bd, dtype=torch.int32, device=self.device), pf[:, 1]])
            seqused = torch.cat([fb.ctx_lens[:Bd], pf[:, 2]])
            bt = torch.cat([fb.block_tables[:Bd], fb.block_tables.index_select(0, pf[:, 3].long())])
        else:
            qlens = torch.ones(Bd, dtype=torch.int32, device=self.device)
            seqused = fb.ctx_lens[:Bd]
            bt = fb.block_tables[:Bd]
        cu = torch.zeros(qlens.numel() + 1, dtype=torch.int32, device=self.device)
        cu[1:] = torch.cumsum(qlens, 0)
        max_q = T if S_pf else 1
        max_k = fb.block_tables.shape[1] * 16
        slots = fb.slots[:T]
        for li, L in enumerate(self.w.layers):
            x = ref.rmsnorm(h, L.in_norm.float(), cfg.rms_eps)[0].to(torch.bfloat16)
            qkv = F.linear(x, L.w_qkv, L.b_qkv)
            q = qkv[:, :hq * D].view(T, hq, D)
            k = qkv[:, hq * D:(hq + hkv) * D].view(T, hkv, D)
            v = qkv[:, (hq + hkv) * D:].reshape(T, hkv, D)
            q = self._rope(q, pos)
            k = self._rope(k, pos)
            kc = k_caches[li].permute(0, 2, 1, 3)  # [blocks, 16, heads, D] view of the pages
            vc = v_caches[li].permute(0, 2, 1, 3)
            self.vops.reshape_and_cache_flash(k, v, kc, vc, slots, "auto", self.k_scale, self.v_scale)
            attn = self.fa(q, kc, vc, max_seqlen_q=max_q, cu_seqlens_q=cu, max_seqlen_k=max_k, seqused_k=seqused,
                           softmax_scale=self.scale, causal=True, block_table=bt, fa_version=2)
            o = F.linear(attn.reshape(T, hq * D), L.w_o)
            h = h + self._all_reduce(o).float()
            x = ref.rmsnorm(h, L.post_norm.float(), cfg.rms_eps)[0].to(torch.bfloat16)
            gu = F.linear(x, L.w_gu)
            Fl = gu.shape[1] // 2
            gate, up = gu.view(T, -1, 2, 128)[:, :, 0].reshape(T, Fl), gu.view(T, -1, 2, 128)[:, :, 1].reshape(T, Fl)
            act = (F.silu(gate.float()) * up.float()).to(torch.bfloat16)
            d = F.linear(act, L.w_down)
            h = h + self._all_reduce(d).float()
        xs = ref.rmsnorm(h.index_select(0, fb.logits_idx), self.w.final_norm.float(), cfg.rms_eps)[0]
        return F.linear(xs.to(torch.bfloat16), self.w.lm_head[:cfg.vocab_size]).float()

    @staticmethod
    def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
               out: torch.Tensor, rep_penalty: torch.Tensor, counts: torch.Tensor, slots: torch.Tensor) -> None:
        """Repetition penalty over the slot's counts, temperature, top-k (the
        batch's largest k), top-p, multinomial draw; greedy rows take argmax."""
        R = logits.shape[0]
        c = counts.index_select(0, slots.long())
        pen = rep_penalty[:, None]
        pl = torch.where(logits > 0, logits / pen.pow(c), logits * pen.pow(c))
        pl = torch.where(c > 0, pl, logits)
        greedy = temperature <= 0
        t = torch.where(greedy, torch.ones_like(temperature), temperature)
        kmax = 1024
        vals, idx = torch.topk(pl / t[:, None], kmax, dim=-1)
        k = torch.where(top_k > 0, top_k, torch.full_like(top_k, kmax)).clamp(max=kmax)
        keep = torch.arange(kmax, device=logits.device)[None, :] < k[:, None]
        vals = torch.where(keep, vals, torch.full_like(vals, float("-inf")))
        probs = torch.softmax(vals, dim=-1)
        cum = torch.cumsum(probs, dim=-1)
        probs = torch.where(cum - probs < top_p[:, None], probs, torch.zeros_like(probs))
        draw = torch.multinomial(probs / probs.sum(-1, keepdim=True), 1)[:, 0]
        tok = idx.gather(1, draw[:, None])[:, 0]
        tok = torch.where(greedy, pl.argmax(-1), tok)
        out[:R].copy_(tok.to(torch.int32))
