"""Functional wrappers over the sm_100a kernels.

Every function here launches kernels from ``kapsl_sdk_b200._cuda`` on the
current CUDA stream.  Plain fp32 PyTorch restatements of the same math live in
:mod:`kapsl_sdk_b200.ops.reference`; the CPU backend and the numerics tests use
them as the oracle.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .._ext import cuda_ops

EPI_PLAIN, EPI_BIAS, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2, 3

_err_bufs: dict[int, torch.Tensor] = {}


def error_buffer(device: torch.device) -> torch.Tensor:
    """Per-device int32[16] status words written by kernels whose bounded
    waits time out (0 = ok).  Read with :func:`check_errors`."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _err_bufs.get(idx)
    if buf is None:
        buf = torch.zeros(16, dtype=torch.int32, device=device)
        _err_bufs[idx] = buf
    return buf


# Status codes the kernels record in the error buffer when a bounded wait runs out
# (or a size check fails); 0 = ok.
DEVICE_ERRORS = {
    1: "decode attention: a KV page load did not arrive within its wait limit",
    2: "prefill attention: a KV page load did not arrive within its wait limit",
    **{c: "GEMM pipeline wait ran out (1-SM kernel)" for c in range(10, 14)},
    **{c: "GEMM pipeline wait ran out (2-SM kernel)" for c in range(20, 24)},
    30: "tensor-parallel reduction (push): a peer missed barrier 1",
    31: "tensor-parallel reduction (push): a peer missed barrier 2",
    32: "tensor-parallel reduction (pull): a peer missed barrier 1",
    33: "tensor-parallel reduction (pull): a peer missed barrier 2",
    34: "tensor-parallel reduction + norm (pull): a peer missed barrier 1",
    35: "tensor-parallel reduction + norm (pull): a peer missed barrier 2",
    36: "tensor-parallel row reduction: a peer's partial rows did not arrive",
    37: "tensor-parallel row reduction: an owner's normed rows did not arrive",
    38: "tensor-parallel row reduction (LL): a peer's partial rows did not arrive",
    39: "NVLink flag probe: the peer's flag did not arrive",
    40: "MoE permute: expert rows exceed the sorted buffer",
    41: "MoE combine: a peer missed barrier 1",
    42: "MoE combine: a peer missed barrier 2",
    50: "vocab-parallel sampler: a peer's candidates did not arrive",
    **{c: "Q4_K GEMM pipeline wait ran out" for c in range(60, 67)},
    **{c: "tcgen05 prefill attention pipeline wait ran out" for c in range(71, 79)},
}


def describe_error(code: int) -> str:
    return f"device error {code}: {DEVICE_ERRORS.get(code, 'unknown status')}"


def check_errors(device: torch.device) -> int:
    """Return (and clear) the first non-zero kernel status word on ``device``."""
    buf = error_buffer(device)
    v = int(buf.max().item())
    if v:
        buf.zero_()
    return v


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out = rmsnorm(x [+ residual]) * weight``; with ``residual`` the sum is
    also stored back into ``residual`` (pre-norm residual stream update)."""
    if out is None:
        out = torch.empty_like(x)
    cuda_ops().rmsnorm(out, x, weight, float(eps), residual)
    return out


def rope_kv_write(qkv: torch.Tensor, positions: torch.Tensor, slots: Optional[torch.Tensor], cos_sin: torch.Tensor,
                  k_cache: torch.Tensor, v_cache: torch.Tensor, num_heads: int, num_kv_heads: int,
                  head_dim: int) -> None:
    """Rotate q and k of ``qkv`` in place and write k, v into the paged cache."""
    cuda_ops().rope_kv_write(qkv, positions, slots, cos_sin, k_cache, v_cache, num_heads, num_kv_heads, head_dim)


def silu_mul(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    F = x.shape[1] // 2
    if out is None:
        out = torch.empty(x.shape[0], F, dtype=x.dtype, device=x.device)
    cuda_ops().silu_mul(out, x)
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, vocab_start: int = 0,
              out: Optional[torch.Tensor] = None, src_rows: Optional[torch.Tensor] = None,
              prev_tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rows of ``table`` for ``ids``.  With ``src_rows``: row ``t < len(src_rows)``
    whose ``src_rows[t] >= 0`` looks up ``prev_tokens[src_rows[t]]`` instead of
    ``ids[t]`` (a token the previous step sampled and the host has not read yet)."""
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    cuda_ops().embedding(out, table, ids, int(vocab_start), src_rows, prev_tokens)
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           residual: Optional[torch.Tensor] = None, swiglu: bool = False, out: Optional[torch.Tensor] = None,
           out_dtype: torch.dtype = torch.bfloat16, workspace: Optional[torch.Tensor] = None,
           force_bn: int = 0, force_splits: int = 0) -> torch.Tensor:
    """``out = epilogue(x @ weight.T)`` on the tcgen05 GEMM.

    Exactly one of ``bias`` / ``residual`` / ``swiglu`` selects the fused
    epilogue.  ``residual`` may be the same tensor as ``out`` (in-place
    residual-stream update).  ``swiglu`` expects the gate/up weight interleaved
    in 128-row blocks (see :func:`interleave_gate_up`) and returns [M, N/2].
    """
    if not isinstance(weight, torch.Tensor):
        return _quant_linear(x, weight, bias, residual, swiglu, out, out_dtype, workspace)
    M, N = x.shape[0], weight.shape[0]
    epi = EPI_PLAIN
    if bias is not None:
        epi = EPI_BIAS
    elif residual is not None:
        epi = EPI_RESIDUAL
    elif swiglu:
        epi = EPI_SWIGLU
    ncols = N // 2 if swiglu else N
    if out is None:
        out = torch.empty(M, ncols, dtype=out_dtype, device=x.device)
    if workspace is None:
        workspace = _workspace(x.device)
    cuda_ops().gemm(x, weight, out, epi, bias, residual, workspace, error_buffer(x.device), force_bn, force_splits)
    return out


# Token count and weight rows from which a Q4_K product dequantizes the whole weight
# matrix to bf16 (one memory-bound pass, ~20.5 bits moved per weight) and runs the
# bf16 tcgen05 GEMM, instead of the fused kernel that dequantizes each weight tile
# again for every 256-token tile.  Measured on B200 (ms, fused -> dequant + bf16):
# 2048 x 8192 x 3584 0.135 -> 0.112, 2048 x 57344 x 8192 1.99 -> 1.69, 2048 x 7168 x 8192
# 0.242 -> 0.231; the fused kernel stays ahead at 1024 tokens (0.126 vs 0.143) and on
# narrow products (2048 x 1280 x 8192: 0.067 vs 0.100).
Q4K_DEQUANT_MIN_M = 2048
Q4K_DEQUANT_MIN_N = 4096

_q4k_scratch: dict[int, torch.Tensor] = {}


def _q4k_weight_scratch(device: torch.device, numel: int) -> Optional[torch.Tensor]:
    """Per-device bf16 buffer for a dequantized weight matrix, grown on demand;
    None when it would have to grow while a CUDA graph is being captured."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _q4k_scratch.get(idx)
    if buf is None or buf.numel() < numel:
        if torch.cuda.is_current_stream_capturing():
            return None
        buf = torch.empty(numel, dtype=torch.bfloat16, device=device)
        _q4k_scratch[idx] = buf
    return buf


def _quant_linear(x, weight, bias, residual, swiglu, out, out_dtype, workspace) -> torch.Tensor:
    """``linear`` for a :class:`~kapsl_sdk_b200.quantization.QuantWeight` (Q4_K):
    the fused dequant GEMM, with residual fused; SwiGLU expects the gate and up
    rows concatenated ([gate; up], not interleaved).  From ``Q4K_DEQUANT_MIN_M``
    tokens and ``Q4K_DEQUANT_MIN_N`` weight rows the weight is dequantized into a scratch matrix (gate/up rows written
    in the interleaved SwiGLU layout) and the bf16 GEMM runs with the same
    epilogue."""
    if weight.fmt != "q4_k":
        raise ValueError(f"no fused kernel for weight format {weight.fmt!r}")
    if out_dtype != torch.bfloat16:
        raise ValueError("quantized linear layers produce bf16")
    M, N = x.shape[0], weight.n
    if workspace is None:
        workspace = _workspace(x.device)
    c = cuda_ops()
    err = error_buffer(x.device)
    if M >= Q4K_DEQUANT_MIN_M and N >= Q4K_DEQUANT_MIN_N and (not weight.tiled or N % 128 == 0):
        buf = _q4k_weight_scratch(x.device, N * weight.k)
        if buf is not None:
            w = buf[:N * weight.k].view(N, weight.k)
            half = N // 2 if swiglu and N % 256 == 0 else 0
            c.q4k_dequant_rows(weight.raw, N, weight.k, weight.tiled, half, w)
            if swiglu and half:
                return linear(x, w, swiglu=True, out=out, workspace=workspace)
            if swiglu:
                return silu_mul(linear(x, w, workspace=workspace), out)
            y = linear(x, w, residual=residual, out=out, workspace=workspace)
            if bias is not None:
                y.add_(bias)
            return y
    if swiglu:
        y = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
        c.gemm_q4k(x, weight.raw, y, weight.k, None, workspace, 0, weight.tiled, err)
        return silu_mul(y, out)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    c.gemm_q4k(x, weight.raw, out, weight.k, residual, workspace, 0, weight.tiled, err)
    if bias is not None:
        out.add_(bias)
    return out


_ws: dict[int, torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int = 64 << 20) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _ws.get(idx)
    if w is None or w.numel() * 4 < nbytes:
        w = torch.empty(nbytes // 4, dtype=torch.float32, device=device)
        _ws[idx] = w
    return w


def workspace(device: torch.device) -> torch.Tensor:
    """The per-device fp32 GEMM workspace (split-K partials)."""
    return _workspace(device)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = 128) -> torch.Tensor:
    """[F, d] gate and up -> [2F, d] with alternating 128-row blocks
    (gate_0, up_0, gate_1, up_1, ...), the layout the SwiGLU epilogue reads."""
    F, d = gate.shape
    assert F % block == 0, "intermediate size must be a multiple of 128"
    g = gate.view(F // block, block, d)
    u = up.view(F // block, block, d)
    return torch.stack([g, u], dim=1).reshape(2 * F, d).contiguous()


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                     ctx_lens: torch.Tensor, num_heads: int, num_kv_heads: int, scale: Optional[float] = None,
                     out: Optional[torch.Tensor] = None, num_splits: int = 0,
                     scratch: Optional[tuple[torch.Tensor, torch.Tensor]] = None,
                     max_ctx: Optional[int] = None) -> torch.Tensor:
    """Paged decode attention (one query token per row of ``q``)."""
    B = q.shape[0]
    D = 128
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, num_heads * D, dtype=q.dtype, device=q.device)
    ops = cuda_ops()
    if num_splits <= 0:
        mc = int(max_ctx) if max_ctx is not None else int(block_tables.shape[1]) * 16
        num_splits = int(ops.decode_num_splits(B, num_kv_heads, mc))
    po = pl = None
    if num_splits > 1:
        if scratch is None:
            po = torch.empty(B * num_heads * num_splits * D, dtype=torch.float32, device=q.device)
            pl = torch.empty(B * num_heads * num_splits, dtype=torch.float32, device=q.device)
        else:
            po, pl = scratch
    ops.decode_attention(q, k_cache, v_cache, block_tables, ctx_lens, out, num_heads, num_kv_heads, float(scale),
                         num_splits, po, pl, error_buffer(q.device))
    return out


def prefill_work(q_lens: list[int], tile: int = 64) -> list[tuple[int, int]]:
    """Work list of (sequence, first query row) tiles for :func:`prefill_attention`."""
    work = []
    for s, n in enumerate(q_lens):
        for t0 in range(0, n, tile):
            work.append((s, t0))
    return work


def prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, work: torch.Tensor,
                      seq_info: torch.Tensor, block_tables: torch.Tensor, num_heads: int, num_kv_heads: int,
                      out: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
    """Chunked-prefill attention.  ``seq_info[s] = (q_start, q_len, ctx_len, bt_row)``;
    the chunk's tokens sit at positions ``ctx_len - q_len .. ctx_len - 1``."""
    if scale is None:
        scale = 1.0 / math.sqrt(128)
    cuda_ops().prefill_attention(q, k_cache, v_cache, work, seq_info, block_tables, out, num_heads, num_kv_heads,
                                 float(scale), error_buffer(q.device))
    return out


def prefill_attention_tc(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, work: torch.Tensor,
                         seq_info: torch.Tensor, block_tables: torch.Tensor, num_heads: int, num_kv_heads: int,
                         out: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
    """:func:`prefill_attention` on the tcgen05 kernel; ``work`` from
    ``prefill_work(q_lens, tile=prefill_tc_tile(num_heads, num_kv_heads))``."""
    if scale is None:
        scale = 1.0 / math.sqrt(128)
    cuda_ops().prefill_attention_tc(q, k_cache, v_cache, work, seq_info, block_tables, out, num_heads, num_kv_heads,
                                    float(scale), error_buffer(q.device))
    return out


def prefill_tc_tile(num_heads: int, num_kv_heads: int) -> int:
    """Query tokens per CTA of the tcgen05 prefill kernel: its 128 MMA rows hold
    every query head of one KV head for floor(128 / group) tokens."""
    return 128 // (num_heads // num_kv_heads)


SAMPLE_MAX_TOP_K = 1024  # top_k above this (or 0, with T > 0) takes the whole-vocabulary path


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           rng_state: torch.Tensor, out: torch.Tensor, rep_penalty: Optional[torch.Tensor] = None,
           counts: Optional[torch.Tensor] = None, slots: Optional[torch.Tensor] = None,
           occ: Optional[torch.Tensor] = None, occ_n: Optional[torch.Tensor] = None,
           full_scratch: Optional[torch.Tensor] = None, full_ctas: int = 0) -> torch.Tensor:
    """Sample one token per row of fp32 ``logits`` (modified in place).

    ``rng_state`` (int64 LCG states), ``counts`` (per-id occurrence counts for
    the repetition penalty) and ``occ`` / ``occ_n`` (each slot's list of ids
    that occurred, so the penalty touches only those logits) are per-sequence
    tables indexed by ``slots[row]`` (or by the row itself when ``slots`` is
    None).  Rows with T > 0 and top_k 0 or > 1024 are sampled over the whole
    vocabulary when ``full_scratch`` (:func:`sample_full_scratch`) is given."""
    cuda_ops().sample(logits, temperature, top_k, top_p, rep_penalty, counts, slots, rng_state, out, occ, occ_n, 0,
                      logits.shape[1], full_scratch, int(full_ctas), [], [], 0, 0, None, 0,
                      error_buffer(logits.device))
    return out


def sample_full_scratch(vocab: int, device, ctas: int = 32) -> torch.Tensor:
    """Scratch for ``ctas`` rows sampled over the whole vocabulary at once."""
    n = int(cuda_ops().sample_full_scratch_bytes(vocab, ctas))
    return torch.empty(n, dtype=torch.uint8, device=device)


def count_tokens(counts: torch.Tensor, rows: torch.Tensor, ids: torch.Tensor, occ: Optional[torch.Tensor] = None,
                 occ_n: Optional[torch.Tensor] = None) -> None:
    """``counts[rows[i], ids[i]] += 1``; a first occurrence also appends the id to
    ``occ[rows[i]]`` (length ``occ_n[rows[i]]``)."""
    cuda_ops().count_tokens(counts, rows, ids, occ, occ_n)


# ------------------------------------------------------------ mixture of experts
def moe_route(x: torch.Tensor, w_router: torch.Tensor, top_k: int, renormalize: bool = True,
              ids: Optional[torch.Tensor] = None, weights: Optional[torch.Tensor] = None):
    """Router logits ``x @ w_router.T`` -> (expert ids int32 [T, k], weights fp32 [T, k])."""
    T = x.shape[0]
    if ids is None:
        ids = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    if weights is None:
        weights = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    cuda_ops().moe_route(x, w_router, top_k, renormalize, ids, weights)
    return ids, weights


def moe_permute(ids: torch.Tensor, num_experts: int, e_lo: int, e_local: int, max_rows: int, seg: torch.Tensor,
                pos: torch.Tensor, mtiles: torch.Tensor, src: torch.Tensor) -> None:
    """Stable expert sort of the [T, k] assignments (segments padded to 128 rows)."""
    T, k = ids.shape
    cuda_ops().moe_permute(ids, T, k, num_experts, e_lo, e_local, max_rows, seg, pos, mtiles, src,
                           error_buffer(ids.device))


def moe_gather(x: torch.Tensor, src: torch.Tensor, mtiles: torch.Tensor, xs: torch.Tensor) -> None:
    cuda_ops().moe_gather(x, src, mtiles, xs)


def grouped_linear(xs: torch.Tensor, w: torch.Tensor, n_per_group: int, mtiles: torch.Tensor,
                   out: torch.Tensor, swiglu: bool = False, splits: int = 1, bn: int = 0,
                   workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-expert GEMM over expert-sorted rows: tile i of ``xs`` times expert
    ``mtiles[1 + i]`` of ``w`` ([groups * n_per_group, K])."""
    groups = w.shape[0] // n_per_group
    if splits > 1 and workspace is None:
        workspace = _workspace(xs.device, splits * xs.shape[0] * n_per_group * 4)
    cuda_ops().grouped_gemm(xs, w, out, n_per_group, groups, mtiles, 3 if swiglu else 0, bn, splits, workspace,
                            error_buffer(xs.device))
    return out


def moe_combine(y_ptrs: list[int], hidden_ptrs: list[int], flag_ptrs: list[int], rank: int, ids: torch.Tensor,
                weights: torch.Tensor, pos: torch.Tensor, seg: torch.Tensor, e_local: int, cols: int, ld_y: int,
                ld_h: int, rows_per_rank: int, epoch: Optional[torch.Tensor] = None,
                timeout_ns: int = 5_000_000_000) -> None:
    """Weighted top-k combine + residual; with peers (len(y_ptrs) > 1) each wait on
    a peer's flag gives up after ``timeout_ns`` and records error 41 / 42."""
    T, k = ids.shape
    cuda_ops().moe_combine(y_ptrs, hidden_ptrs, flag_ptrs, rank, ids, weights, pos, seg, T, k, e_local, cols, ld_y,
                           ld_h, rows_per_rank, epoch, error_buffer(ids.device), int(timeout_ns))
