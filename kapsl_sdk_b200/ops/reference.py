"""Plain fp32 PyTorch restatements of every kernel in :mod:`kapsl_sdk_b200.ops`.

These are the numerics oracle for the CUDA kernels and the math of the CPU
backend.  The sampler follows the reference runtime's semantics exactly
(crates/kapsl-llm/src/engine.rs:5817-5927, penalty at engine.rs:3104-3123).
"""
from __future__ import annotations

import math
from typing import Iterable, Optional, Sequence

import numpy as np
import torch

MASK64 = (1 << 64) - 1


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None):
    xf = x.float()
    if residual is not None:
        xf = xf + residual.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return xf * torch.rsqrt(var + eps) * weight.float(), xf


def rope_inv_freq(head_dim: int, theta: float, scaling: Optional[dict] = None) -> tuple:
    """Rotary inverse frequencies (float64 [head_dim / 2]) and the factor that
    scales cos/sin, for the RoPE scaling of HF ``rope_scaling`` / GGUF metadata:

    * ``linear``: every frequency divided by ``factor`` (position interpolation);
    * ``llama3``: wavelengths above ``original_max_position_embeddings /
      low_freq_factor`` divided by ``factor``, below ``... / high_freq_factor``
      kept, a linear blend in between (Llama 3.1);
    * ``yarn``: per-dimension blend of extrapolated and interpolated
      frequencies over the ramp between the dimensions that rotate
      ``beta_fast`` and ``beta_slow`` times in the original context, with
      cos/sin scaled by ``attention_factor`` (default 0.1 ln(factor) + 1)
      (Peng et al., "YaRN", 2023);
    * ``freq_factors``: explicit per-frequency divisors (GGUF ``rope_freqs``).
    Scalings that depend on the live sequence length (dynamic NTK, LongRoPE)
    are refused rather than approximated by a fixed table."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if not scaling:
        return inv, 1.0
    kind = scaling.get("rope_type", scaling.get("type", "default"))
    if kind in ("default", None):
        return inv, 1.0
    factor = float(scaling.get("factor", 1.0))
    if kind == "linear":
        return inv / factor, 1.0
    if kind == "freq_factors":
        f = torch.as_tensor(scaling["factors"], dtype=torch.float64)
        if f.numel() != inv.numel():
            raise ValueError(f"rope frequency factors: {f.numel()} values for {inv.numel()} frequencies")
        return inv / f, 1.0
    if kind == "llama3":
        orig = float(scaling["original_max_position_embeddings"])
        lo, hi = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
        wavelen = 2 * math.pi / inv
        smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        blended = (1 - smooth) * inv / factor + smooth * inv
        out = torch.where(wavelen > orig / lo, inv / factor, blended)
        return torch.where(wavelen < orig / hi, inv, out), 1.0
    if kind == "yarn":
        orig = float(scaling.get("original_max_position_embeddings", 4096))
        beta_fast, beta_slow = float(scaling.get("beta_fast", 32.0)), float(scaling.get("beta_slow", 1.0))
        attn = scaling.get("attention_factor")
        if attn is None:
            mscale = float(scaling.get("mscale", 1.0) or 1.0)
            mscale_all = float(scaling.get("mscale_all_dim", 0.0) or 0.0)

            def m(s, k):
                return 1.0 if s <= 1 else 0.1 * k * math.log(s) + 1.0

            attn = m(factor, mscale) / m(factor, mscale_all) if mscale_all else m(factor, 1.0)

        def corr_dim(rotations):
            return head_dim * math.log(orig / (rotations * 2 * math.pi)) / (2 * math.log(theta))

        low = corr_dim(beta_fast)
        high = corr_dim(beta_slow)
        if scaling.get("truncate", True):
            low, high = math.floor(low), math.ceil(high)
        low, high = max(low, 0), min(high, head_dim - 1)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(head_dim // 2, dtype=torch.float64) - low) / (high - low)).clamp(0.0, 1.0)
        extrap = 1 - ramp
        return inv / factor * (1 - extrap) + inv * extrap, float(attn)
    raise ValueError(f"RoPE scaling {kind!r} depends on the live sequence length; not supported")


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, device=None, scaling: Optional[dict] = None
                 ) -> torch.Tensor:
    """[max_pos, head_dim] fp32 table: cos in the first half, sin in the second
    (``scaling``: see :func:`rope_inv_freq`)."""
    inv, attn = rope_inv_freq(head_dim, theta, scaling)
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return (torch.cat([f.cos(), f.sin()], dim=1) * attn).float().to(device)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """x: [T, H, D] -> rotated (NeoX rotate-half convention)."""
    D = x.shape[-1]
    half = D // 2
    cs = cos_sin[positions.long()].float()
    c, s = cs[:, None, :half], cs[:, None, half:]
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    F = x.shape[-1] // 2
    g, u = x[..., :F].float(), x[..., F:].float()
    return g * torch.sigmoid(g) * u


def gelu_tanh_mul(x: torch.Tensor) -> torch.Tensor:
    """GeGLU with the tanh approximation of GELU: gelu(g) * u over [g | u]."""
    F = x.shape[-1] // 2
    g, u = x[..., :F].float(), x[..., F:].float()
    return torch.nn.functional.gelu(g, approximate="tanh") * u


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal_offset: int,
              softcap: float = 0.0, window: int = 0) -> torch.Tensor:
    """q: [Sq, Hq, D]; k, v: [Sk, Hkv, D]; query i sees keys <= causal_offset + i
    (and, with ``window``, only the last ``window`` of them); ``softcap`` > 0
    maps the scaled logits through cap * tanh(s / cap)."""
    Sq, Hq, D = q.shape
    Sk, Hkv, _ = k.shape
    g = Hq // Hkv
    kk = k.float().repeat_interleave(g, dim=1)
    vv = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk) * scale
    if softcap > 0:
        s = torch.tanh(s / softcap) * softcap
    qi = torch.arange(Sq)[:, None] + causal_offset
    ki = torch.arange(Sk)[None, :]
    masked = ki > qi
    if window:
        masked = masked | (qi - ki >= window)
    s = s.masked_fill(masked[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vv)


def gather_paged(cache: torch.Tensor, block_table: Sequence[int], length: int) -> torch.Tensor:
    """cache [blocks, Hkv, BS, D] -> contiguous [length, Hkv, D]."""
    BS = cache.shape[2]
    nb = (length + BS - 1) // BS
    blocks = cache[torch.as_tensor(list(block_table[:nb]), dtype=torch.long)]  # [nb, Hkv, BS, D]
    return blocks.permute(0, 2, 1, 3).reshape(nb * BS, cache.shape[1], cache.shape[3])[:length]


# ---------------------------------------------------------------- sampling
def fnv1a64(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h ^= b
        h = (h * 0x100000001B3) & MASK64
    return h


def splitmix64(x: int) -> int:
    z = (x + 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def seed_state(seed: Optional[int], request_id: str, seq_id: int) -> int:
    """rng = splitmix64((seed ?? fnv1a(request_id)) ^ seq_id * golden) (engine.rs:2349-2358)."""
    base = seed if seed is not None else fnv1a64(request_id.encode())
    return splitmix64((base ^ ((seq_id * 0x9E3779B97F4A7C15) & MASK64)) & MASK64)


def next_f32(state: int) -> tuple[float, int]:
    state = (state * 6364136223846793005 + 1) & MASK64
    val = np.float32(state >> 32)
    return float(np.float32(val / np.float32(4294967295.0))), state


def apply_repetition_penalty(logits: np.ndarray, token_ids: Iterable[int], penalty: float) -> np.ndarray:
    out = logits.astype(np.float32).copy()
    p = np.float32(penalty)
    for t in token_ids:
        if 0 <= t < out.shape[0]:
            v = out[t]
            out[t] = v / p if v > 0 else v * p
    return out


def sample_next_token(logits: np.ndarray, temperature: float, top_k: int, top_p: float,
                      state: int) -> tuple[int, int]:
    """Reference sampler: returns (token, new rng state)."""
    logits = np.asarray(logits, dtype=np.float32)
    if logits.size == 0:
        return 0, state
    if temperature <= 0.0:
        m = logits.max()
        return int(np.nonzero(logits == m)[0][-1]), state  # last max wins (Iterator::max_by)
    k = logits.size if top_k == 0 else min(top_k, logits.size)
    k = max(k, 1)
    scaled = (logits / np.float32(temperature)).astype(np.float32)
    order = np.lexsort((np.arange(scaled.size), -scaled))[:k]  # descending, lower index first
    top = [(int(i), np.float32(scaled[i])) for i in order]
    tp = min(max(top_p, 0.0), 1.0)
    if tp < 1.0 and len(top) > 1:
        mx = top[0][1]
        ex = [np.float32(np.exp(np.float32(l - mx))) for _, l in top]
        s = np.float32(0.0)
        for e in ex:
            s = np.float32(s + e)
        cum = np.float32(0.0)
        cutoff = len(top)
        for i, e in enumerate(ex):
            cum = np.float32(cum + np.float32(e / s))
            if cum >= np.float32(tp):
                cutoff = i + 1
                break
        top = top[:cutoff]
    mx = top[0][1]
    ex = [np.float32(np.exp(np.float32(l - mx))) for _, l in top]
    s = np.float32(0.0)
    for e in ex:
        s = np.float32(s + e)
    u, state = next_f32(state)
    draw = np.float32(np.float32(u) * s)
    for (idx, _), e in zip(top, ex):
        if draw <= e:
            return idx, state
        draw = np.float32(draw - e)
    return top[0][0], state
