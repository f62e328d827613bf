"""Llama-family decoder (Llama / Qwen2 / Mixtral attention stack) on the sm_100a kernels.

One ``CausalLM`` instance per GPU.  Under tensor parallelism the weights are
Megatron-sharded (column-parallel QKV and gate/up, row-parallel o/down,
vocab-parallel embedding and lm_head) and the per-layer reduction goes through
:class:`kapsl_sdk_b200.parallel.tp.TPComm` (NCCL baseline or the fused
NVLink kernels).

Reference counterpart: the reference runs the whole transformer inside ONNX
Runtime sessions (crates/kapsl-llm/src/engine.rs:2885-2890, 3567) and has no
model code of its own.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Optional

import torch

from .. import ops
from ..ops import reference as ref
from .config import ModelConfig


# Chunked-prefill attention on tcgen05 (attention_tc.cu) by default: checked against the fp32
# oracle and 3-10% faster than the mma.sync kernel on 2048- and 8192-token chunks.
PREFILL_TC_DEFAULT = True


def _prefill(model, qkv, k_cache, v_cache, fb, attn) -> None:
    fn = ops.prefill_attention_tc if model.prefill_tc else ops.prefill_attention
    fn(qkv, k_cache, v_cache, fb.pf_work, fb.pf_seq_info, fb.block_tables, model.hq, model.hkv, attn, model.scale)


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    w_qkv: torch.Tensor            # [(hq + 2*hkv) * D, d]  (local heads)
    b_qkv: Optional[torch.Tensor]  # [(hq + 2*hkv) * D]
    w_o: torch.Tensor              # [d, hq * D]
    w_gu: Optional[torch.Tensor] = None    # [2F_local, d], gate/up interleaved in 128-row blocks
    w_down: Optional[torch.Tensor] = None  # [d, F_local]
    # MoE
    w_router: Optional[torch.Tensor] = None        # [E, d]
    w_experts_gu: Optional[torch.Tensor] = None    # [E_local, 2F, d] interleaved
    w_experts_down: Optional[torch.Tensor] = None  # [E_local, d, F]


@dataclass
class ModelWeights:
    embed: torch.Tensor      # [V_local, d]
    lm_head: torch.Tensor    # [V_local, d]
    final_norm: torch.Tensor
    layers: list = field(default_factory=list)
    vocab_start: int = 0
    heads_local: int = 0
    kv_heads_local: int = 0
    ffn_local: int = 0


@dataclass
class ShardPlan:
    """How a model is split over ``tp`` ranks.

    ``q_pad`` extra (zero) query heads per KV group make the head count
    divisible by ``tp`` when it is not (e.g. 28 heads over 8 ranks: each of the
    4 KV groups is padded from 7 to 8 query heads and every KV head is held by
    2 ranks).  Padded heads have zero q weights and zero o_proj columns, so the
    result is unchanged.
    """
    tp: int
    rank: int
    group: int          # real query heads per KV head
    group_pad: int      # padded query heads per KV head
    kv_heads_local: int
    kv_head_start: int
    heads_local: int
    q_slot_start: int   # first padded query slot of this rank

    @staticmethod
    def make(cfg: ModelConfig, tp: int, rank: int) -> "ShardPlan":
        g = cfg.num_heads // cfg.num_kv_heads
        hq_pad = cfg.num_heads
        gp = g
        if cfg.num_heads % tp != 0:
            # pad each group so that padded heads split evenly and each rank's
            # slice stays inside one KV group
            gp = g
            while (cfg.num_kv_heads * gp) % tp != 0 or (tp > cfg.num_kv_heads and gp % (tp // cfg.num_kv_heads) != 0):
                gp += 1
            hq_pad = cfg.num_kv_heads * gp
        heads_local = hq_pad // tp
        if tp <= cfg.num_kv_heads:
            assert cfg.num_kv_heads % tp == 0, "kv heads must divide over tp"
            kvl = cfg.num_kv_heads // tp
            kvs = rank * kvl
        else:
            assert tp % cfg.num_kv_heads == 0, "tp must be a multiple of kv heads"
            kvl = 1
            kvs = rank // (tp // cfg.num_kv_heads)
        return ShardPlan(tp=tp, rank=rank, group=g, group_pad=gp, kv_heads_local=kvl, kv_head_start=kvs,
                         heads_local=heads_local, q_slot_start=rank * heads_local)

    def local_q_heads(self) -> list[int]:
        """Original head index for each local query slot (-1 = padding)."""
        out = []
        for s in range(self.q_slot_start, self.q_slot_start + self.heads_local):
            kv, j = divmod(s, self.group_pad)
            out.append(kv * self.group + j if j < self.group else -1)
        return out


def ffn_shard_size(cfg: ModelConfig, tp: int) -> int:
    """Per-rank FFN width: F / tp rounded up to the GEMM tile (128; 256 for Q4_K,
    whose blocks span 256 inputs).  Ranks past F hold zero gate/up rows and zero
    down columns (e.g. Qwen2.5-7B's 18944 over 8 ranks: 2368 -> 2432)."""
    align = 256 if cfg.weight_format == "q4_k" else 128
    return -(-cfg.intermediate_size // (tp * align)) * align


def vocab_slice(vocab: int, tp: int) -> int:
    """Vocabulary columns per rank of the vocab-parallel lm_head: ceil(V / tp)
    rounded up to the GEMM's 128-row tile (Qwen2.5-7B over 8 ranks: 19072)."""
    return -(-vocab // (tp * 128)) * 128 if tp > 1 else vocab


def _pad_rows(w: torch.Tensor, n: int) -> torch.Tensor:
    return w if w.shape[0] == n else torch.cat([w, w.new_zeros(n - w.shape[0], *w.shape[1:])], 0)


def _shard_rows(w: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    n = w.shape[0] // tp
    return w[rank * n:(rank + 1) * n]


def _shard_cols(w: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    n = w.shape[1] // tp
    return w[:, rank * n:(rank + 1) * n]


def shard_layer(cfg: ModelConfig, plan: ShardPlan, full: dict, device, dtype=torch.bfloat16) -> LayerWeights:
    """Cut one layer's full (unsharded, HF-layout) tensors for ``plan.rank``.

    ``full`` keys: q, k, v ([heads*D, d]), q_b, k_b, v_b (optional), o ([d, heads*D]),
    gate, up ([F, d]), down ([d, F]), in_norm, post_norm; MoE: router [E, d],
    experts_gate/up [E, F, d], experts_down [E, d, F].
    """
    D = cfg.head_dim
    tp, r = plan.tp, plan.rank
    qh = plan.local_q_heads()
    q = full["q"].view(cfg.num_heads, D, -1)
    qrows = [q[h] if h >= 0 else torch.zeros_like(q[0]) for h in qh]
    kv0, kvn = plan.kv_head_start, plan.kv_heads_local
    k = full["k"].view(cfg.num_kv_heads, D, -1)[kv0:kv0 + kvn]
    v = full["v"].view(cfg.num_kv_heads, D, -1)[kv0:kv0 + kvn]
    w_qkv = torch.cat([torch.stack(qrows).reshape(-1, cfg.hidden_size), k.reshape(-1, cfg.hidden_size),
                       v.reshape(-1, cfg.hidden_size)], 0)
    b_qkv = None
    if full.get("q_b") is not None:
        qb = full["q_b"].view(cfg.num_heads, D)
        qbl = [qb[h] if h >= 0 else torch.zeros_like(qb[0]) for h in qh]
        kb = full["k_b"].view(cfg.num_kv_heads, D)[kv0:kv0 + kvn]
        vb = full["v_b"].view(cfg.num_kv_heads, D)[kv0:kv0 + kvn]
        b_qkv = torch.cat([torch.stack(qbl).reshape(-1), kb.reshape(-1), vb.reshape(-1)])
    o = full["o"].view(cfg.hidden_size, cfg.num_heads, D)
    ocols = [o[:, h] if h >= 0 else torch.zeros_like(o[:, 0]) for h in qh]
    w_o = torch.stack(ocols, 1).reshape(cfg.hidden_size, -1)
    lw = LayerWeights(in_norm=full["in_norm"].to(device, dtype), post_norm=full["post_norm"].to(device, dtype),
                      w_qkv=w_qkv.to(device, dtype).contiguous(),
                      b_qkv=b_qkv.to(device, dtype).contiguous() if b_qkv is not None else None,
                      w_o=w_o.to(device, dtype).contiguous())
    if cfg.is_moe:
        E = cfg.num_experts
        assert E % tp == 0 or tp % E == 0
        lw.w_router = full["router"].to(device, dtype).contiguous()
        # expert parallel: experts split over ranks
        el = max(E // tp, 1)
        e0 = (r * el) % E
        gu = [ops.interleave_gate_up(full["experts_gate"][e], full["experts_up"][e]) for e in range(e0, e0 + el)]
        lw.w_experts_gu = torch.stack(gu).to(device, dtype).contiguous()
        lw.w_experts_down = full["experts_down"][e0:e0 + el].to(device, dtype).contiguous()
    else:
        Fp = ffn_shard_size(cfg, tp) * tp
        gate = _shard_rows(_pad_rows(full["gate"], Fp), r, tp)
        up = _shard_rows(_pad_rows(full["up"], Fp), r, tp)
        if cfg.weight_format == "q4_k":
            lw.w_gu = torch.cat([gate, up], 0).to(device, dtype).contiguous()  # [gate; up] for the Q4_K path
        else:
            lw.w_gu = ops.interleave_gate_up(gate, up).to(device, dtype).contiguous()
        lw.w_down = _shard_cols(_pad_rows(full["down"].T, Fp).T, r, tp).to(device, dtype).contiguous()
    if cfg.weight_format == "q4_k":
        from ..quantization import quantize_q4_k

        lw.w_qkv = quantize_q4_k(lw.w_qkv)
        lw.w_o = quantize_q4_k(lw.w_o)
        if lw.w_gu is not None:
            lw.w_gu = quantize_q4_k(lw.w_gu)
            lw.w_down = quantize_q4_k(lw.w_down)
    elif cfg.weight_format != "bf16":
        raise ValueError(f"unsupported weight format {cfg.weight_format!r}")
    return lw


def random_layer(cfg: ModelConfig, layer: int, gen: torch.Generator, device, std: float = 0.02) -> dict:
    """Full-size random tensors for one layer, N(0, std) (norms = 1)."""
    d, F, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim

    def rn(*shape):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.bfloat16) * std

    full = {
        "q": rn(cfg.num_heads * D, d), "k": rn(cfg.num_kv_heads * D, d), "v": rn(cfg.num_kv_heads * D, d),
        "o": rn(d, cfg.num_heads * D),
        "in_norm": torch.ones(d, device=device, dtype=torch.bfloat16),
        "post_norm": torch.ones(d, device=device, dtype=torch.bfloat16),
    }
    if cfg.qk_norm:
        full["q_norm"] = torch.ones(D, device=device, dtype=torch.bfloat16) + rn(D) * 10
        full["k_norm"] = torch.ones(D, device=device, dtype=torch.bfloat16) + rn(D) * 10
    if cfg.qkv_bias:
        full["q_b"] = rn(cfg.num_heads * D)
        full["k_b"] = rn(cfg.num_kv_heads * D)
        full["v_b"] = rn(cfg.num_kv_heads * D)
    if cfg.is_moe:
        E = cfg.num_experts
        full["router"] = rn(E, d)
        full["experts_gate"] = rn(E, F, d)
        full["experts_up"] = rn(E, F, d)
        full["experts_down"] = rn(E, d, F)
    else:
        full["gate"] = rn(F, d)
        full["up"] = rn(F, d)
        full["down"] = rn(d, F)
    return full


def random_full_weights(cfg: ModelConfig, device, seed: int = 0, std: float = 0.02):
    """Yields ("embed", t), ("lm_head", t), then ("layer", full_dict) per layer:
    the unsharded random tensors, drawn in a fixed order from ``seed``."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    d, V = cfg.hidden_size, cfg.vocab_size
    emb = torch.randn(V, d, generator=gen, device=device, dtype=torch.bfloat16) * std
    yield "embed", emb
    head = emb if cfg.tie_embeddings else torch.randn(V, d, generator=gen, device=device, dtype=torch.bfloat16) * std
    yield "lm_head", head
    for layer in range(cfg.num_layers):
        yield "layer", random_layer(cfg, layer, gen, device, std)


def weights_from_full(cfg: ModelConfig, full_iter, device, tp: int = 1, rank: int = 0,
                      layers: Optional[range] = None) -> ModelWeights:
    """Shard a stream of full tensors (see :func:`random_full_weights`) for one rank;
    ``layers`` keeps only a pipeline stage's layer range."""
    plan = ShardPlan.make(cfg, tp, rank)
    V, d = cfg.vocab_size, cfg.hidden_size
    # the embedding is replicated (a lookup of T rows); the lm_head is held whole on
    # every rank, padded with zero rows to tp equal vocabulary slices: a step
    # multiplies only this rank's slice and the sampler merges the ranks'
    # candidates (the whole matrix serves steps that sample over every id)
    vl, v0 = V, 0
    vpad = vocab_slice(V, tp) * tp
    w = ModelWeights(embed=None, lm_head=None, final_norm=torch.ones(d, device=device, dtype=torch.bfloat16),
                     vocab_start=v0, heads_local=plan.heads_local, kv_heads_local=plan.kv_heads_local,
                     ffn_local=ffn_shard_size(cfg, tp) if not cfg.is_moe else cfg.intermediate_size)
    layer_idx = 0
    for kind, t in full_iter:
        if kind == "embed":
            w.embed = t[v0:v0 + vl].to(device, torch.bfloat16).contiguous()
        elif kind == "lm_head":
            w.lm_head = _pad_rows(t[v0:v0 + vl].to(device, torch.bfloat16), vpad).contiguous()
        elif kind == "final_norm":
            w.final_norm = t.to(device, torch.bfloat16).contiguous()
        else:
            li = layer_idx
            layer_idx += 1
            if layers is None or li in layers:
                w.layers.append(shard_layer(cfg, plan, t, device))
    return w


def random_weights(cfg: ModelConfig, device, tp: int = 1, rank: int = 0, seed: int = 0,
                   std: float = 0.02, layers: Optional[range] = None) -> ModelWeights:
    """Random-init weights N(0, std) from ``seed``; every rank draws the same full
    tensors layer by layer and keeps its shard, so TP results match TP1."""
    return weights_from_full(cfg, random_full_weights(cfg, device, seed, std), device, tp, rank, layers)


@dataclass
class ForwardBatch:
    """Device inputs of one model step (tokens of decode rows first)."""
    input_ids: torch.Tensor      # int32 [T]
    positions: torch.Tensor      # int32 [T]
    slots: torch.Tensor          # int64 [T]
    block_tables: torch.Tensor   # int32 [S, max_blocks]  (decode sequences first)
    ctx_lens: torch.Tensor       # int32 [S]
    logits_idx: torch.Tensor     # int64 [R]
    num_tokens: int
    num_decode: int
    max_decode_ctx: int = 0
    pf_work: Optional[torch.Tensor] = None      # int32 [n, 2]
    pf_seq_info: Optional[torch.Tensor] = None  # int32 [S_pf, 4]
    decode_splits: int = 0
    # tokens still on the device: row t < len(src_rows) with src_rows[t] >= 0
    # embeds prev_tokens[src_rows[t]] (the previous step's sample) instead of input_ids[t]
    src_rows: Optional[torch.Tensor] = None     # int32 [n]
    prev_tokens: Optional[torch.Tensor] = None  # int32 [R_prev]


class CausalLM:
    """GPU decoder over a paged KV cache, one instance per rank."""

    def __init__(self, cfg: ModelConfig, weights: ModelWeights, device, tp_comm=None, moe=None, stage=None):
        if cfg.cpu_only:
            raise ValueError(f"{cfg.arch} layers (q/k norms, GeGLU, soft-capping or sliding windows) run on the "
                             "CPU backend only")
        self.cfg = cfg
        self.w = weights
        self.device = torch.device(device)
        self.tp = tp_comm
        self.moe = moe
        self.stage = stage  # PipelineStage: ``weights.layers`` are this stage's layers only
        self.hq = weights.heads_local
        self.hkv = weights.kv_heads_local
        self.D = cfg.head_dim
        self.scale = 1.0 / math.sqrt(self.D)
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, cfg.head_dim, cfg.rope_theta, device=self.device,
                                         scaling=cfg.rope_scaling)
        self.qkv_width = (self.hq + 2 * self.hkv) * self.D
        W = self.tp_size
        # chunked-prefill attention: the tcgen05 kernel (head group packed into the 128
        # MMA rows, floor(128 / g) query tokens per work item) or the mma.sync kernel
        # (64-token work items); KAPSL_PREFILL_TC=0/1 overrides the default
        env = os.environ.get("KAPSL_PREFILL_TC")
        self.prefill_tc = (env == "1") if env is not None else PREFILL_TC_DEFAULT
        g = self.hq // max(self.hkv, 1)
        self.prefill_tile = (128 // g) if self.prefill_tc and 0 < g <= 128 else 64
        self.vocab_slice = vocab_slice(cfg.vocab_size, W)
        self.vocab_start = (tp_comm.rank if W > 1 else 0) * self.vocab_slice

    def configure_tp(self, max_tokens: int, sample_rows: int = 0) -> None:
        if self.tp is not None and self.tp.world_size > 1:
            self.tp.configure(max_tokens, self.cfg.hidden_size, sample_rows=sample_rows)
        if self.moe is not None:
            self.moe.configure(max_tokens)

    @property
    def tp_size(self) -> int:
        return 1 if self.tp is None else self.tp.world_size

    def forward(self, fb: ForwardBatch, k_caches: list, v_caches: list, full_vocab: bool = True) -> torch.Tensor:
        """Logits (fp32) of the rows ``fb.logits_idx``: every vocabulary column, or
        with tensor parallelism and ``full_vocab=False`` only this rank's slice
        (columns [vocab_start, vocab_start + vocab_slice))."""
        cfg = self.cfg
        T = fb.num_tokens
        Bd = fb.num_decode
        tp = self.tp_size > 1
        h = self.tp.residual_stream(T) if tp else None  # symmetric memory in fused TP mode
        st = self.stage
        if st is not None and not st.first:  # later pipeline stage: the previous stage's hidden state
            hin = st.recv_hidden(T, cfg.hidden_size, torch.bfloat16, self.device)
            h = hin if h is None else h.copy_(hin)
        else:
            h = ops.embedding(fb.input_ids[:T], self.w.embed, self.w.vocab_start, out=h, src_rows=fb.src_rows,
                              prev_tokens=fb.prev_tokens)
        attn = torch.empty(T, self.hq * self.D, dtype=torch.bfloat16, device=self.device)
        if tp and self.moe is None and st is None and self.tp.fused_norm:
            return self._forward_sharded(fb, k_caches, v_caches, h, attn, full_vocab)
        x = torch.empty_like(h)
        for li, L in enumerate(self.w.layers):
            ops.rmsnorm(h, L.in_norm, cfg.rms_eps, out=x)
            qkv = ops.linear(x, L.w_qkv, bias=L.b_qkv)
            ops.rope_kv_write(qkv, fb.positions, fb.slots, self.cos_sin, k_caches[li], v_caches[li], self.hq,
                              self.hkv, self.D)
            if Bd > 0:
                ops.decode_attention(qkv[:Bd], k_caches[li], v_caches[li], fb.block_tables[:Bd], fb.ctx_lens[:Bd],
                                     self.hq, self.hkv, self.scale, out=attn[:Bd], num_splits=fb.decode_splits,
                                     max_ctx=fb.max_decode_ctx)
            if T > Bd:
                _prefill(self, qkv, k_caches[li], v_caches[li], fb, attn)
            if not tp:
                ops.linear(attn, L.w_o, residual=h, out=h)
            else:
                self.tp.row_parallel_residual(attn, L.w_o, h)
            ops.rmsnorm(h, L.post_norm, cfg.rms_eps, out=x)
            if self.moe is not None:
                self.moe.forward(x, L, h)  # adds the routed experts' output into h
            elif not tp:
                g = ops.linear(x, L.w_gu, swiglu=True)
                ops.linear(g, L.w_down, residual=h, out=h)
            else:
                g = ops.linear(x, L.w_gu, swiglu=True)
                self.tp.row_parallel_residual(g, L.w_down, h)
        if st is not None and not st.last:
            st.send_hidden(h[:T].clone())
            return None
        xs = h.index_select(0, fb.logits_idx)
        xs = ops.rmsnorm(xs, self.w.final_norm, cfg.rms_eps)
        return self._lm_head(xs, full_vocab)

    def _lm_head(self, xs: torch.Tensor, full_vocab: bool) -> torch.Tensor:
        if self.tp_size > 1 and not full_vocab:
            head = self.w.lm_head[self.vocab_start:self.vocab_start + self.vocab_slice]
        else:
            head = self.w.lm_head[:self.cfg.vocab_size]
        return ops.linear(xs, head, out_dtype=torch.float32)

    def _forward_sharded(self, fb: ForwardBatch, k_caches: list, v_caches: list, h: torch.Tensor,
                         attn: torch.Tensor, full_vocab: bool) -> torch.Tensor:
        """Fused tensor-parallel layer loop: every row-parallel GEMM is followed by
        one kernel that reduces the rows this rank owns, adds them to its shard
        of the residual stream, applies the next RMSNorm (the next layer's input
        norm, or the final norm after the last layer) and stores the normed rows
        into every rank's input buffer.  No separate norm launches and no full
        residual copies."""
        cfg = self.cfg
        T, Bd = fb.num_tokens, fb.num_decode
        layers = self.w.layers
        x = self.tp.norm_input(T)
        ops.rmsnorm(h, layers[0].in_norm, cfg.rms_eps, out=x)  # embedding rows are on every rank
        for li, L in enumerate(layers):
            qkv = ops.linear(x, L.w_qkv, bias=L.b_qkv)
            ops.rope_kv_write(qkv, fb.positions, fb.slots, self.cos_sin, k_caches[li], v_caches[li], self.hq,
                              self.hkv, self.D)
            if Bd > 0:
                ops.decode_attention(qkv[:Bd], k_caches[li], v_caches[li], fb.block_tables[:Bd], fb.ctx_lens[:Bd],
                                     self.hq, self.hkv, self.scale, out=attn[:Bd], num_splits=fb.decode_splits,
                                     max_ctx=fb.max_decode_ctx)
            if T > Bd:
                _prefill(self, qkv, k_caches[li], v_caches[li], fb, attn)
            x = self.tp.row_parallel_norm(attn, L.w_o, h, L.post_norm, cfg.rms_eps)
            g = ops.linear(x, L.w_gu, swiglu=True)
            nxt = layers[li + 1].in_norm if li + 1 < len(layers) else self.w.final_norm
            x = self.tp.row_parallel_norm(g, L.w_down, h, nxt, cfg.rms_eps)
        return self._lm_head(x.index_select(0, fb.logits_idx), full_vocab)


def reference_forward(cfg: ModelConfig, full_layers: list, embed: torch.Tensor, lm_head: torch.Tensor,
                      final_norm: torch.Tensor, tokens: list[int]) -> torch.Tensor:
    """fp32 dense forward over one sequence (oracle for the paged GPU path).
    Returns logits [len(tokens), V]."""
    D = cfg.head_dim
    cs = ref.rope_cos_sin(cfg.max_position, D, cfg.rope_theta, scaling=cfg.rope_scaling)
    ids = torch.tensor(tokens)
    pos = torch.arange(len(tokens))
    h = embed.float()[ids]
    for full in full_layers:
        x, _ = ref.rmsnorm(h, full["in_norm"], cfg.rms_eps)
        q = x @ full["q"].float().T
        k = x @ full["k"].float().T
        v = x @ full["v"].float().T
        if full.get("q_b") is not None:
            q = q + full["q_b"].float()
            k = k + full["k_b"].float()
            v = v + full["v_b"].float()
        q, k = q.view(-1, cfg.num_heads, D), k.view(-1, cfg.num_kv_heads, D)
        if full.get("q_norm") is not None:  # Qwen3: per-head RMSNorm before RoPE
            q = ref.rmsnorm(q, full["q_norm"], cfg.rms_eps)[0]
            k = ref.rmsnorm(k, full["k_norm"], cfg.rms_eps)[0]
        q = ref.apply_rope(q, pos, cs)
        k = ref.apply_rope(k, pos, cs)
        v = v.view(-1, cfg.num_kv_heads, D)
        a = ref.attention(q, k, v, 1.0 / math.sqrt(D), 0).reshape(len(tokens), -1)
        h = h + a @ full["o"].float().T
        x, _ = ref.rmsnorm(h, full["post_norm"], cfg.rms_eps)
        if cfg.is_moe:
            logits_r = x @ full["router"].float().T
            p = torch.softmax(logits_r, -1)
            topv, topi = p.topk(cfg.experts_per_token, -1)
            topv = topv / topv.sum(-1, keepdim=True)
            out = torch.zeros_like(x)
            for e in range(cfg.num_experts):
                sel = (topi == e)
                rows = sel.any(-1).nonzero().flatten()
                if rows.numel() == 0:
                    continue
                wgt = (topv * sel).sum(-1)[rows]
                xe = x[rows]
                g = xe @ full["experts_gate"][e].float().T
                u = xe @ full["experts_up"][e].float().T
                y = (g * torch.sigmoid(g) * u) @ full["experts_down"][e].float().T
                out[rows] += wgt[:, None] * y
            h = h + out
        else:
            g = x @ full["gate"].float().T
            u = x @ full["up"].float().T
            h = h + (g * torch.sigmoid(g) * u) @ full["down"].float().T
    x, _ = ref.rmsnorm(h, final_norm, cfg.rms_eps)
    return x @ lm_head.float().T
