"""GGUF model files: reading, block dequantization, Q4_K quantization, writing.

Reference: GGUF models are served by llama.cpp (crates/kapsl-llm/src/gguf_backend.rs);
here GGUF is parsed with the ``gguf`` package's reader/writer and the tensors
are turned into this runtime's weight layout.  The quantized block formats are
the GGML ones (they have to match to read real files):

* Q8_0: 32 values, f16 scale ``d`` + 32 x int8; v = d * q
* Q4_K: 256 values in 8 sub-blocks of 32; f16 ``d`` and ``dmin``, 12 bytes of
  packed 6-bit (scale, min) pairs, 128 bytes of 4-bit quants; v = d*sc_j*q - dmin*m_j.
  Quants of sub-blocks 2c and 2c+1 share bytes 32c..32c+31 (low / high nibble).
* Q6_K: 256 values; 128 bytes of low 4 bits, 64 bytes of high 2 bits, 16 int8
  sub-block scales, f16 ``d``; v = d * sc * (q - 32).
* Q4_0 / Q4_1 / Q5_0 / Q5_1 (32 values), Q2_K / Q3_K / Q5_K (256 values): dequantized
  at load by the functions below (checked against the gguf package's dequantizers);
  any other GGML type goes through the gguf package's NumPy dequantizer.

Llama-architecture files store q/k projections permuted for interleaved rotary
pairs; they are permuted back to the rotate-half layout the RoPE kernel uses.
"""
from __future__ import annotations

import os
from typing import Optional

import numpy as np
import torch

from ..models.config import ModelConfig

QK_K = 256
Q4_K_BYTES = 144
Q6_K_BYTES = 210
Q8_0_BYTES = 34


# ------------------------------------------------------------ dequantization
def _q4k_scale_min(sc: np.ndarray):
    """sc: [nb, 12] uint8 -> scales, mins [nb, 8] (6-bit each)."""
    s = np.empty((sc.shape[0], 8), np.uint8)
    m = np.empty((sc.shape[0], 8), np.uint8)
    s[:, :4] = sc[:, 0:4] & 63
    m[:, :4] = sc[:, 4:8] & 63
    s[:, 4:] = (sc[:, 8:12] & 0xF) | ((sc[:, 0:4] >> 6) << 4)
    m[:, 4:] = (sc[:, 8:12] >> 4) | ((sc[:, 4:8] >> 6) << 4)
    return s, m


def dequant_q4_k(raw: np.ndarray) -> np.ndarray:
    b = raw.reshape(-1, Q4_K_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    s, m = _q4k_scale_min(b[:, 4:16])
    qs = b[:, 16:144].reshape(-1, 4, 32)
    q = np.empty((b.shape[0], 8, 32), np.float32)
    q[:, 0::2] = qs & 0xF
    q[:, 1::2] = qs >> 4
    out = d[:, :, None] * s[:, :, None].astype(np.float32) * q - dmin[:, :, None] * m[:, :, None].astype(np.float32)
    return out.reshape(-1)


def dequant_q6_k(raw: np.ndarray) -> np.ndarray:
    b = raw.reshape(-1, Q6_K_BYTES)
    ql = b[:, 0:128].astype(np.int32)
    qh = b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)
    out = np.empty((b.shape[0], 256), np.float32)
    for half in range(2):
        L = ql[:, half * 64:(half + 1) * 64]
        H = qh[:, half * 32:(half + 1) * 32]
        S = sc[:, half * 8:(half + 1) * 8]
        base = half * 128
        q1 = (L[:, :32] & 0xF) | ((H & 3) << 4)
        q2 = (L[:, 32:] & 0xF) | (((H >> 2) & 3) << 4)
        q3 = (L[:, :32] >> 4) | (((H >> 4) & 3) << 4)
        q4 = (L[:, 32:] >> 4) | (((H >> 6) & 3) << 4)
        for j, q in enumerate((q1, q2, q3, q4)):
            idx = np.arange(32) // 16
            scl = S[:, idx + 2 * j]
            out[:, base + 32 * j:base + 32 * j + 32] = d * scl * (q - 32)  # d: [nb, 1]
    return out.reshape(-1)


def dequant_q8_0(raw: np.ndarray) -> np.ndarray:
    b = raw.reshape(-1, Q8_0_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (d * q).reshape(-1)


def _f16(b: np.ndarray, at: int) -> np.ndarray:
    """[nb, 1] float32 from the f16 at byte offset `at` of each block."""
    return b[:, at:at + 2].copy().view(np.float16).astype(np.float32)


def _nibbles32(qs: np.ndarray) -> np.ndarray:
    """[nb, 16] bytes -> [nb, 32] quants: value j < 16 is the low nibble of byte j,
    value 16 + j its high nibble (the legacy 32-value block order)."""
    return np.concatenate([qs & 0xF, qs >> 4], axis=1).astype(np.float32)


def _high_bits32(qh: np.ndarray) -> np.ndarray:
    """[nb, 4] bytes (a little-endian u32) -> [nb, 32] bits, bit j for value j."""
    return np.unpackbits(qh, axis=1, bitorder="little").astype(np.float32)


def dequant_q4_0(raw: np.ndarray) -> np.ndarray:
    """32 values: f16 d, 16 bytes of 4-bit quants; v = d * (q - 8)."""
    b = raw.reshape(-1, 18)
    return (_f16(b, 0) * (_nibbles32(b[:, 2:18]) - 8)).reshape(-1)


def dequant_q4_1(raw: np.ndarray) -> np.ndarray:
    """32 values: f16 d, f16 m, 16 bytes of 4-bit quants; v = d * q + m."""
    b = raw.reshape(-1, 20)
    return (_f16(b, 0) * _nibbles32(b[:, 4:20]) + _f16(b, 2)).reshape(-1)


def dequant_q5_0(raw: np.ndarray) -> np.ndarray:
    """32 values: f16 d, 4 bytes of fifth bits, 16 bytes of low nibbles; v = d * (q - 16)."""
    b = raw.reshape(-1, 22)
    q = _nibbles32(b[:, 6:22]) + 16 * _high_bits32(b[:, 2:6])
    return (_f16(b, 0) * (q - 16)).reshape(-1)


def dequant_q5_1(raw: np.ndarray) -> np.ndarray:
    """32 values: f16 d, f16 m, 4 bytes of fifth bits, 16 bytes of low nibbles; v = d * q + m."""
    b = raw.reshape(-1, 24)
    q = _nibbles32(b[:, 8:24]) + 16 * _high_bits32(b[:, 4:8])
    return (_f16(b, 0) * q + _f16(b, 2)).reshape(-1)


def dequant_q5_k(raw: np.ndarray) -> np.ndarray:
    """256 values in 8 sub-blocks of 32: f16 d, f16 dmin, 12 bytes of 6-bit (scale,
    min) pairs packed as in Q4_K, 32 bytes of fifth bits, 128 bytes of low nibbles.
    Sub-blocks 2c and 2c+1 share nibble bytes 32c..32c+31 (low / high nibble); the
    fifth bit of value l of sub-block s is bit s of high byte l."""
    b = raw.reshape(-1, 176)
    d, dmin = _f16(b, 0), _f16(b, 2)
    sc, mn = _q4k_scale_min(b[:, 4:16])
    qh = b[:, 16:48]
    qs = b[:, 48:176].reshape(-1, 4, 32)
    q = np.empty((b.shape[0], 8, 32), np.int32)
    q[:, 0::2] = qs & 0xF
    q[:, 1::2] = qs >> 4
    q |= ((qh[:, None, :] >> np.arange(8, dtype=np.uint8)[None, :, None]) & 1).astype(np.int32) << 4
    out = (d[:, :, None] * sc[:, :, None].astype(np.float32)) * q.astype(np.float32) - \
        dmin[:, :, None] * mn[:, :, None].astype(np.float32)
    return out.reshape(-1)


def dequant_q2_k(raw: np.ndarray) -> np.ndarray:
    """256 values in 16 groups of 16: 16 bytes of (4-bit scale | 4-bit min << 4), 64
    bytes of 2-bit quants, f16 d, f16 dmin; v = d * scale * q - dmin * min.  Each half
    of 128 values reads 32 quant bytes four times (shifts 0, 2, 4, 6); group g of a
    half takes bytes 16 * (g % 2) .. + 15 at shift 2 * (g // 2)."""
    b = raw.reshape(-1, 84)
    scale, mn = (b[:, 0:16] & 0xF).astype(np.float32), (b[:, 0:16] >> 4).astype(np.float32)
    d, dmin = _f16(b, 80), _f16(b, 82)
    qs = b[:, 16:80].reshape(-1, 2, 2, 16)  # [nb, half, byte group, 16]
    q = np.empty((b.shape[0], 2, 8, 16), np.float32)
    for g in range(8):
        q[:, :, g] = (qs[:, :, g % 2] >> (2 * (g // 2))) & 3
    q = q.reshape(-1, 16, 16)
    return (d[:, :, None] * scale[:, :, None] * q - dmin[:, :, None] * mn[:, :, None]).reshape(-1)


def _q3k_scales(sc: np.ndarray) -> np.ndarray:
    """[nb, 12] bytes -> [nb, 16] signed scales (6 bits each, biased by 32): the low
    4 bits of scales 0-7 / 8-15 are the low / high nibbles of bytes 0-7, the top 2
    bits come from bytes 8-11 (2 bits per scale, shifts 0, 2, 4, 6 for scale groups
    of four)."""
    lo = np.concatenate([sc[:, 0:8] & 0xF, sc[:, 0:8] >> 4], axis=1).astype(np.int32)
    hi = np.empty((sc.shape[0], 16), np.int32)
    for k in range(4):
        hi[:, 4 * k:4 * k + 4] = (sc[:, 8:12] >> (2 * k)) & 3
    return ((hi << 4) | lo) - 32


def dequant_q3_k(raw: np.ndarray) -> np.ndarray:
    """256 values in 16 groups of 16: 32 bytes of high-bit masks, 64 bytes of 2-bit
    quants, 12 bytes of 6-bit scales, f16 d; v = d * scale * (q - 4 * (1 - h)) where q
    is the 2-bit quant and h its mask bit.  Quant bytes are laid out as in Q2_K; the
    mask bit of value l (0-31) in the j-th 32-value run of the block is bit j of mask
    byte l."""
    b = raw.reshape(-1, 110)
    hm = b[:, 0:32]
    qs = b[:, 32:96].reshape(-1, 2, 2, 16)
    scale = _q3k_scales(b[:, 96:108]).astype(np.float32)
    d = _f16(b, 108)
    q = np.empty((b.shape[0], 2, 8, 16), np.int32)
    for g in range(8):
        q[:, :, g] = (qs[:, :, g % 2] >> (2 * (g // 2))) & 3
    q = q.reshape(-1, 8, 32)  # 32-value runs: run r covers groups 2r, 2r+1
    h = ((hm[:, None, :] >> np.arange(8, dtype=np.uint8)[None, :, None]) & 1).astype(np.int32)
    q = (q - 4 * (1 - h)).reshape(-1, 16, 16).astype(np.float32)
    return (d[:, :, None] * scale[:, :, None] * q).reshape(-1)


# -------------------------------------------------------------- quantization
def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    """fp32 [n * 256] -> Q4_K bytes.  Per 32-value sub-block: min = max(0, -min(x)),
    scale = (max(x) + min) / 15; the 8 scales and mins are then coded as 6-bit
    multiples of the super-block ``d = max(scale) / 63`` and ``dmin = max(min) / 63``."""
    x = np.asarray(x, np.float32).reshape(-1, 8, 32)
    nb = x.shape[0]
    lo = np.minimum(x.min(-1), 0.0)
    hi = x.max(-1)
    mins = -lo
    scales = (hi - lo) / 15.0
    d = scales.max(-1) / 63.0
    dmin = mins.max(-1) / 63.0
    d16 = d.astype(np.float16)
    dm16 = dmin.astype(np.float16)
    dq = np.where(d16 > 0, d16.astype(np.float32), 1.0)
    dmq = np.where(dm16 > 0, dm16.astype(np.float32), 1.0)
    sc = np.clip(np.rint(scales / dq[:, None]), 0, 63).astype(np.uint8)
    mn = np.clip(np.rint(mins / dmq[:, None]), 0, 63).astype(np.uint8)
    eff_s = d16.astype(np.float32)[:, None] * sc
    eff_m = dm16.astype(np.float32)[:, None] * mn
    q = np.where(eff_s[:, :, None] > 0, np.rint((x + eff_m[:, :, None]) / np.where(eff_s > 0, eff_s, 1)[:, :, None]), 0)
    q = np.clip(q, 0, 15).astype(np.uint8)
    out = np.zeros((nb, Q4_K_BYTES), np.uint8)
    out[:, 0:2] = d16.reshape(-1, 1).view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dm16.reshape(-1, 1).view(np.uint8).reshape(nb, 2)
    p = np.zeros((nb, 12), np.uint8)
    p[:, 0:4] = (sc[:, :4] & 63) | ((sc[:, 4:] >> 4) << 6)
    p[:, 4:8] = (mn[:, :4] & 63) | ((mn[:, 4:] >> 4) << 6)
    p[:, 8:12] = (sc[:, 4:] & 0xF) | ((mn[:, 4:] & 0xF) << 4)
    out[:, 4:16] = p
    qq = q.reshape(nb, 4, 2, 32)
    out[:, 16:] = (qq[:, :, 0] | (qq[:, :, 1] << 4)).reshape(nb, 128)
    return out.reshape(-1)


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    """fp32 [n * 256] -> Q6_K bytes.  Per 16-value group: scale = max|x| / 32
    (signed by the value of largest magnitude, so it maps to -32); the 16 scales
    are coded as int8 multiples of ``d = max|scale| / 127``; quants are
    round(x / (d * sc)) + 32 clipped to 0..63."""
    x = np.asarray(x, np.float32).reshape(-1, 16, 16)
    nb = x.shape[0]
    idx = np.abs(x).argmax(-1)
    vmax = np.take_along_axis(x, idx[..., None], -1)[..., 0]
    scales = -vmax / 32.0
    d = np.abs(scales).max(-1) / 127.0
    d16 = d.astype(np.float16)
    dq = np.where(d16 > 0, d16.astype(np.float32), 1.0)
    sc = np.clip(np.rint(scales / dq[:, None]), -127, 127).astype(np.int8)
    eff = d16.astype(np.float32)[:, None] * sc
    q = np.where(eff[:, :, None] != 0, np.rint(x / np.where(eff != 0, eff, 1)[:, :, None]), 0) + 32
    q = np.clip(q, 0, 63).astype(np.uint8).reshape(nb, 2, 4, 32)  # [block, half, quarter, 32]
    out = np.zeros((nb, Q6_K_BYTES), np.uint8)
    lo, hi = q & 0xF, q >> 4
    for h in range(2):
        out[:, h * 64:h * 64 + 32] = lo[:, h, 0] | (lo[:, h, 2] << 4)
        out[:, h * 64 + 32:h * 64 + 64] = lo[:, h, 1] | (lo[:, h, 3] << 4)
        out[:, 128 + h * 32:128 + h * 32 + 32] = hi[:, h, 0] | (hi[:, h, 1] << 2) | (hi[:, h, 2] << 4) | (hi[:, h, 3] << 6)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d16.reshape(-1, 1).view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


# ------------------------------------------------------------------ reading
def _permute_back(w: np.ndarray, n_head: int) -> np.ndarray:
    """Undo the interleaved-rotary permutation of llama q/k rows."""
    rows, cols = w.shape
    hd = rows // n_head
    return w.reshape(n_head, hd // 2, 2, cols).swapaxes(1, 2).reshape(rows, cols)


def _permute(w: np.ndarray, n_head: int) -> np.ndarray:
    rows, cols = w.shape
    hd = rows // n_head
    return w.reshape(n_head, 2, hd // 2, cols).swapaxes(1, 2).reshape(rows, cols)


def tensor_to_numpy(t) -> np.ndarray:
    """A gguf ReaderTensor -> fp32 array in (rows, cols) order."""
    from gguf import GGMLQuantizationType as Q

    shape = tuple(int(x) for x in reversed(t.shape))  # GGUF lists ne0 (innermost) first
    raw = np.asarray(t.data)
    tt = t.tensor_type
    if tt == Q.F32:
        a = raw.astype(np.float32)
    elif tt == Q.F16:
        a = raw.view(np.float16).astype(np.float32)
    elif tt == Q.BF16:
        a = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    elif tt == Q.Q8_0:
        a = dequant_q8_0(raw.view(np.uint8))
    elif tt == Q.Q4_K:
        a = dequant_q4_k(raw.view(np.uint8))
    elif tt == Q.Q6_K:
        a = dequant_q6_k(raw.view(np.uint8))
    elif tt in (Q.Q4_0, Q.Q4_1, Q.Q5_0, Q.Q5_1, Q.Q2_K, Q.Q3_K, Q.Q5_K):
        a = {Q.Q4_0: dequant_q4_0, Q.Q4_1: dequant_q4_1, Q.Q5_0: dequant_q5_0, Q.Q5_1: dequant_q5_1,
             Q.Q2_K: dequant_q2_k, Q.Q3_K: dequant_q3_k, Q.Q5_K: dequant_q5_k}[tt](raw.view(np.uint8))
    else:
        # remaining GGML formats (IQ*, TQ*, ...) through the gguf package's NumPy dequantizers
        from gguf import quants

        try:
            a = quants.dequantize(raw, tt)
        except NotImplementedError:
            raise ValueError(f"unsupported GGUF tensor type {tt.name} for {t.name}") from None
    return a.reshape(shape)


def _field(reader, key, default=None):
    f = reader.fields.get(key)
    if f is None:
        return default
    try:
        v = f.contents()
    except Exception:
        v = f.parts[f.data[0]] if f.data else default
        if hasattr(v, "tolist"):
            v = v.tolist()
            if isinstance(v, list) and len(v) == 1:
                v = v[0]
    return v


GGUF_ARCHS = ("llama", "qwen2", "qwen3", "phi3", "gemma", "gemma2")


def gguf_config(reader) -> ModelConfig:
    arch = _field(reader, "general.architecture", "llama")
    if arch not in GGUF_ARCHS:
        raise ValueError(f"GGUF architecture {arch!r} is not supported (supported: {', '.join(GGUF_ARCHS)})")
    p = lambda k, d=None: _field(reader, f"{arch}.{k}", d)
    heads = int(p("attention.head_count", 32))
    hidden = int(p("embedding_length", 4096))
    tokens = _field(reader, "tokenizer.ggml.tokens")
    vocab = int(p("vocab_size", len(tokens) if tokens is not None else 32000))
    return ModelConfig(
        name=_field(reader, "general.name", arch) or arch,
        arch=arch if arch in ("qwen2", "qwen3", "gemma", "gemma2") else "llama",
        qk_norm=arch == "qwen3", **_gguf_gemma(reader, arch, hidden, int(p("attention.key_length", hidden // heads))),
        vocab_size=vocab, hidden_size=hidden, intermediate_size=int(p("feed_forward_length", 4 * hidden)),
        num_layers=int(p("block_count", 32)), num_heads=heads, num_kv_heads=int(p("attention.head_count_kv", heads)),
        head_dim=int(p("attention.key_length", hidden // heads)), rope_theta=float(p("rope.freq_base", 10000.0)),
        rms_eps=float(p("attention.layer_norm_rms_epsilon", 1e-5)), qkv_bias=arch == "qwen2",
        max_position=min(int(p("context_length", 4096)), 4096),
        bos_token_id=_field(reader, "tokenizer.ggml.bos_token_id", 1),
        eos_token_id=_field(reader, "tokenizer.ggml.eos_token_id", 2),
        rope_scaling=_gguf_rope_scaling(reader, arch),
    )


def _gguf_gemma(reader, arch: str, hidden: int, head_dim: int) -> dict:
    """Gemma options from GGUF (norm weights there already include the +1)."""
    if arch not in ("gemma", "gemma2"):
        return {}
    out = dict(act="gelu_tanh", embed_scale=hidden ** 0.5, tie_embeddings=True)
    if arch == "gemma2":
        window = int(_field(reader, "gemma2.attention.sliding_window", 0) or 0)
        out.update(attn_softcap=float(_field(reader, "gemma2.attn_logit_softcapping", 0.0) or 0.0),
                   final_softcap=float(_field(reader, "gemma2.final_logit_softcapping", 0.0) or 0.0),
                   attn_scale=float(_field(reader, "gemma2.attention.scale", head_dim ** -0.5)),
                   sliding_window=window, sliding_pattern=2 if window else 0)
    return out


def _gguf_rope_scaling(reader, arch: str) -> Optional[dict]:
    """RoPE scaling from GGUF: per-frequency divisors stored as the
    ``rope_freqs.weight`` tensor (Llama 3.1 exports), else the
    ``{arch}.rope.scaling.*`` keys (linear / yarn)."""
    for t in reader.tensors:
        if t.name in ("rope_factors_long.weight", "rope_factors_short.weight"):
            raise ValueError("LongRoPE (rope_factors_long/short) depends on the live sequence length; not supported")
        if t.name == "rope_freqs.weight":
            return {"rope_type": "freq_factors", "factors": [float(v) for v in np.asarray(t.data).reshape(-1)]}
    kind = _field(reader, f"{arch}.rope.scaling.type")
    if kind in (None, "none"):
        return None
    rs = {"rope_type": str(kind), "factor": float(_field(reader, f"{arch}.rope.scaling.factor", 1.0))}
    orig = _field(reader, f"{arch}.rope.scaling.original_context_length")
    if orig is not None:
        rs["original_max_position_embeddings"] = int(orig)
    return rs


def _q4k_rows(t):
    """A 2-D Q4_K, Q6_K or Q8_0 tensor as kept-packed rows (None for other
    types, and for Q8_0 rows whose length is not a multiple of 256)."""
    from gguf import GGMLQuantizationType as Q

    from ..quantization import Q4KRows, Q6KRows, Q80Rows

    cls = {Q.Q4_K: Q4KRows, Q.Q6_K: Q6KRows, Q.Q8_0: Q80Rows}.get(t.tensor_type)
    if cls is None or len(t.shape) != 2 or int(t.shape[0]) % QK_K:
        return None
    n, k = int(t.shape[1]), int(t.shape[0])
    return cls(np.asarray(t.data).view(np.uint8).reshape(n, k // QK_K * cls.BLOCK), k)


def _row_perm(rows: int, n_head: int) -> np.ndarray:
    """Row order of _permute_back as an index array."""
    return _permute_back(np.arange(rows)[:, None], n_head)[:, 0]


def iter_gguf_full(path: str, cfg: Optional[ModelConfig] = None, keep_q4k: bool = False):
    """Yields the runtime's full-tensor stream (see models.llama.random_full_weights).
    ``keep_q4k``: 2-D Q4_K and Q6_K weights stay packed (``Q4KRows`` / ``Q6KRows``) for the CPU backend."""
    from gguf import GGUFReader

    r = GGUFReader(path)
    cfg = cfg or gguf_config(r)
    T = {t.name: t for t in r.tensors}

    def get(n):
        if keep_q4k:
            q = _q4k_rows(T[n])
            if q is not None:
                return q
        return torch.from_numpy(np.ascontiguousarray(tensor_to_numpy(T[n])))

    def permute(w, n_head):
        if isinstance(w, torch.Tensor):
            return torch.from_numpy(np.ascontiguousarray(_permute_back(w.numpy(), n_head)))
        return w.take(_row_perm(w.n, n_head))

    def split(w, sizes):
        if isinstance(w, torch.Tensor):
            return torch.split(w, sizes, 0)
        out, a = [], 0
        for n in sizes:
            out.append(w.rows(a, a + n))
            a += n
        return out

    permuted = _field(r, "general.architecture", "llama") == "llama"
    emb = torch.from_numpy(np.ascontiguousarray(tensor_to_numpy(T["token_embd.weight"])))
    yield "embed", emb
    yield "lm_head", get("output.weight") if "output.weight" in T else emb
    yield "final_norm", get("output_norm.weight")
    for i in range(cfg.num_layers):
        b = f"blk.{i}."
        if b + "attn_qkv.weight" in T:  # Phi-3: fused [q; k; v]
            q, k, v = split(get(b + "attn_qkv.weight"), [cfg.q_size, cfg.kv_size, cfg.kv_size])
        else:
            q, k, v = get(b + "attn_q.weight"), get(b + "attn_k.weight"), get(b + "attn_v.weight")
        if permuted:
            q = permute(q, cfg.num_heads)
            k = permute(k, cfg.num_kv_heads)
        full = {"q": q, "k": k, "v": v, "o": get(b + "attn_output.weight"),
                "in_norm": get(b + "attn_norm.weight"), "post_norm": get(b + "ffn_norm.weight"),
                "down": get(b + "ffn_down.weight")}
        if b + "post_attention_norm.weight" in T:  # Gemma 2 sandwich norms
            full["attn_out_norm"] = get(b + "post_attention_norm.weight")
            full["mlp_out_norm"] = get(b + "post_ffw_norm.weight")
        if b + "ffn_gate.weight" in T:
            full["gate"], full["up"] = get(b + "ffn_gate.weight"), get(b + "ffn_up.weight")
        else:  # Phi-3: ffn_up holds [gate; up]
            gu = get(b + "ffn_up.weight")
            full["gate"], full["up"] = split(gu, [gu.shape[0] // 2, gu.shape[0] // 2])
        if b + "attn_q_norm.weight" in T:  # Qwen3
            full["q_norm"], full["k_norm"] = get(b + "attn_q_norm.weight"), get(b + "attn_k_norm.weight")
        if b + "attn_q.bias" in T:
            full["q_b"], full["k_b"], full["v_b"] = (get(b + "attn_q.bias"), get(b + "attn_k.bias"),
                                                   get(b + "attn_v.bias"))
        yield "layer", full


def gguf_tokenizer(path: str):
    from gguf import GGUFReader

    from ..llm.tokenizer import GGUFTokenizer

    r = GGUFReader(path)
    toks = _field(r, "tokenizer.ggml.tokens")
    if not toks:
        return None
    return GGUFTokenizer(toks, _field(r, "tokenizer.ggml.scores"), _field(r, "tokenizer.ggml.token_type"),
                         _field(r, "tokenizer.ggml.bos_token_id", 1), _field(r, "tokenizer.ggml.eos_token_id", 2),
                         model=str(_field(r, "tokenizer.ggml.model", "llama")),
                         merges=_field(r, "tokenizer.ggml.merges"), pre=_field(r, "tokenizer.ggml.pre"),
                         add_space_prefix=bool(_field(r, "tokenizer.ggml.add_space_prefix", True)))


def load_gguf_model(path: str, device, tp: int = 1, rank: int = 0):
    from gguf import GGUFReader

    from ..models.cpu_model import CPUCausalLM
    from ..models.llama import weights_from_full

    cfg = gguf_config(GGUFReader(path))
    tok = gguf_tokenizer(path)
    dev = torch.device(device)
    # on the CPU backend Q4_K projections stay quantized (KAPSL_CPU_Q4K=0 dequantizes them at load)
    keep = dev.type == "cpu" and os.environ.get("KAPSL_CPU_Q4K", "1") == "1"
    stream = iter_gguf_full(path, cfg, keep_q4k=keep)
    if dev.type == "cpu":
        items = list(stream)
        d = dict((k, v) for k, v in items if k != "layer")
        return cfg, CPUCausalLM(cfg, d["embed"], d["lm_head"], d["final_norm"],
                                [v for k, v in items if k == "layer"]), tok
    gpu_stream = ((k, v.to(dev, torch.bfloat16) if isinstance(v, torch.Tensor)
                   else {kk: vv.to(dev, torch.bfloat16) for kk, vv in v.items()}) for k, v in stream)
    return cfg, weights_from_full(cfg, gpu_stream, dev, tp, rank), tok


# ------------------------------------------------------------------ writing
def synthetic_vocab(n: int) -> tuple:
    """Tokens for a random-init model: <unk>, <s>, </s>, 256 byte tokens, then pieces."""
    toks = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    types = [2, 3, 3] + [6] * 256
    i = 0
    while len(toks) < n:
        toks.append(f"▁t{i}")
        types.append(1)
        i += 1
    return toks[:n], [0.0] * n, types[:n]


def write_gguf_model(path: str, cfg: ModelConfig, full_stream, quant: str = "f32", arch: str = "llama") -> None:
    """Serialize a full-tensor stream as a GGUF file of architecture ``arch``
    ("llama": q/k rows permuted as llama.cpp stores them; "phi3": fused
    attn_qkv and [gate; up] in ffn_up, no permutation).
    ``quant``: "f32", "f16", "q4_k" (2-D weights quantized, norms kept f32) or
    "q4_k_m" (Q4_K with Q6_K for output, attn_v and ffn_down, the mix of
    llama.cpp's Q4_K_M preset applied to every layer), "q8_0", or the legacy
    32-value formats "q4_0" / "q5_1" (written with the gguf package's quantizer)."""
    from gguf import GGMLQuantizationType as Q
    from gguf import GGUFWriter

    if arch not in ("llama", "phi3", "qwen3", "gemma2"):
        raise ValueError(f"cannot write GGUF architecture {arch!r}")
    w = GGUFWriter(path, arch)
    w.add_name(cfg.name)
    w.add_context_length(cfg.max_position)
    w.add_embedding_length(cfg.hidden_size)
    w.add_block_count(cfg.num_layers)
    w.add_feed_forward_length(cfg.intermediate_size)
    w.add_head_count(cfg.num_heads)
    w.add_head_count_kv(cfg.num_kv_heads)
    w.add_rope_freq_base(cfg.rope_theta)
    w.add_layer_norm_rms_eps(cfg.rms_eps)
    w.add_vocab_size(cfg.vocab_size)
    toks, scores, types = synthetic_vocab(cfg.vocab_size)
    w.add_tokenizer_model("llama")
    w.add_token_list(toks)
    w.add_token_scores(scores)
    w.add_token_types(types)
    w.add_bos_token_id(1)
    w.add_eos_token_id(2)

    def put(name, t: torch.Tensor, is_weight: bool):
        a = t.detach().float().cpu().numpy()
        six = quant == "q4_k_m" and (name == "output.weight" or name.endswith((".attn_v.weight", ".ffn_down.weight")))
        if six and is_weight and a.ndim == 2 and a.shape[1] % QK_K == 0:
            w.add_tensor(name, quantize_q6_k(a.reshape(-1)).reshape(a.shape[0], -1), raw_dtype=Q.Q6_K)
        elif quant in ("q8_0", "q4_0", "q5_1") and is_weight and a.ndim == 2 and a.shape[1] % QK_K == 0:
            from gguf import quants

            qt = {"q8_0": Q.Q8_0, "q4_0": Q.Q4_0, "q5_1": Q.Q5_1}[quant]
            w.add_tensor(name, quants.quantize(np.ascontiguousarray(a), qt), raw_dtype=qt)
        elif quant in ("q4_k", "q4_k_m") and is_weight and a.ndim == 2 and a.shape[1] % QK_K == 0:
            # quantized tensors are handed over as [rows, bytes per row]
            w.add_tensor(name, quantize_q4_k(a.reshape(-1)).reshape(a.shape[0], -1), raw_dtype=Q.Q4_K)
        elif quant == "f16" and a.ndim == 2:
            w.add_tensor(name, a.astype(np.float16))
        else:
            w.add_tensor(name, np.ascontiguousarray(a.astype(np.float32)))

    if arch == "gemma2":
        w.add_float32("gemma2.attn_logit_softcapping", cfg.attn_softcap)
        w.add_float32("gemma2.final_logit_softcapping", cfg.final_softcap)
        w.add_uint32("gemma2.attention.sliding_window", cfg.sliding_window)
        w.add_float32("gemma2.attention.scale", cfg.attn_scale or cfg.head_dim ** -0.5)
        w.add_uint32("gemma2.attention.key_length", cfg.head_dim)
    rs = cfg.rope_scaling or {}
    if rs.get("rope_type") == "freq_factors":
        w.add_tensor("rope_freqs.weight", np.asarray(rs["factors"], dtype=np.float32))
    elif rs.get("rope_type") in ("linear", "yarn"):
        w.add_string(f"{arch}.rope.scaling.type", rs["rope_type"])
        w.add_float32(f"{arch}.rope.scaling.factor", float(rs.get("factor", 1.0)))
        if "original_max_position_embeddings" in rs:
            w.add_uint32(f"{arch}.rope.scaling.original_context_length", int(rs["original_max_position_embeddings"]))
    elif rs:
        raise ValueError(f"GGUF cannot store RoPE scaling {rs.get('rope_type')!r}; use frequency factors")

    li = 0
    saw_norm = False
    for kind, t in full_stream:
        if kind == "embed":
            put("token_embd.weight", t, True)
        elif kind == "lm_head":
            put("output.weight", t, True)
        elif kind == "final_norm":
            put("output_norm.weight", t, False)
            saw_norm = True
        else:
            b = f"blk.{li}."
            put(b + "attn_norm.weight", t["in_norm"], False)
            put(b + "ffn_norm.weight", t["post_norm"], False)
            if arch == "phi3":
                put(b + "attn_qkv.weight", torch.cat([t["q"], t["k"], t["v"]], 0), True)
            elif arch == "gemma2":  # unpermuted; norms carry the +1; sandwich norms
                put(b + "attn_q.weight", t["q"], True)
                put(b + "attn_k.weight", t["k"], True)
                put(b + "attn_v.weight", t["v"], True)
                put(b + "post_attention_norm.weight", t["attn_out_norm"], False)
                put(b + "post_ffw_norm.weight", t["mlp_out_norm"], False)
            elif arch == "qwen3":  # stored unpermuted, with per-head q/k norms
                put(b + "attn_q.weight", t["q"], True)
                put(b + "attn_k.weight", t["k"], True)
                put(b + "attn_v.weight", t["v"], True)
                put(b + "attn_q_norm.weight", t["q_norm"], False)
                put(b + "attn_k_norm.weight", t["k_norm"], False)
            else:
                put(b + "attn_q.weight", torch.from_numpy(_permute(t["q"].float().cpu().numpy(), cfg.num_heads)),
                    True)
                put(b + "attn_k.weight", torch.from_numpy(_permute(t["k"].float().cpu().numpy(), cfg.num_kv_heads)),
                    True)
                put(b + "attn_v.weight", t["v"], True)
            put(b + "attn_output.weight", t["o"], True)
            if arch == "phi3":
                put(b + "ffn_up.weight", torch.cat([t["gate"], t["up"]], 0), True)
            else:
                put(b + "ffn_gate.weight", t["gate"], True)
                put(b + "ffn_up.weight", t["up"], True)
            put(b + "ffn_down.weight", t["down"], True)
            li += 1
    if not saw_norm:
        put("output_norm.weight", torch.ones(cfg.hidden_size), False)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
