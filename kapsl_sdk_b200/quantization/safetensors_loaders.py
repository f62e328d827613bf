"""GPTQ / AWQ / INT8 checkpoints from safetensors, with the dequantization math.

Tensor groups (per linear layer ``<name>``):

* GPTQ: ``qweight`` int32 [K/8, N] (8 4-bit values per word along K, low
  nibble first), ``qzeros`` int32 [K/g, N/8] (packed along N), ``scales``
  fp16 [K/g, N], optional ``g_idx`` int32 [K] (group of each input row when
  ``desc_act`` reordered them), optional ``bias``.  w[k, n] = scales[g, n] *
  (q[k, n] - (z[g, n] + zero_offset)), g = g_idx[k] or k // group_size;
  ``zero_offset`` is 1 for checkpoints that store zero - 1 (the common GPTQ
  v1 layout).
* AWQ: ``qweight`` int32 [K, N/8] (packed along N in the interleaved order
  0, 2, 4, 6, 1, 3, 5, 7), ``qzeros`` int32 [K/g, N/8] (same order),
  ``scales`` fp16 [K/g, N]; w[k, n] = scales[g, n] * (q[k, n] - z[g, n]).
* INT8: ``weight`` int8 [N, K] with ``scale`` (fp32) and ``zero_point``
  (int32) scalars; w = scale * (q - zero_point).

``dequantize`` returns the weight as [N, K] (the layout of ``nn.Linear`` and
of this package's GEMMs).  Reference: crates/kapsl-quantization (config.rs:3-30,
tensor.rs:4-35, loader/{gptq,awq,int8}.rs) reads the same tensors but has no
dequantization.
"""
from __future__ import annotations

import glob
import json
import os
from dataclasses import dataclass, field
from typing import Optional

import torch

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)  # nibble slot -> column within each group of 8


@dataclass
class QuantizationConfig:
    quantization_method: str = "int8"  # int8 | gptq | awq
    bits: int = 8
    group_size: int = 128
    desc_act: bool = False
    sym: bool = True

    @classmethod
    def from_dict(cls, d: dict) -> "QuantizationConfig":
        m = (d.get("quantization_method") or d.get("quant_method") or "int8").lower()
        if m not in ("int8", "gptq", "awq"):
            raise ValueError(f"unknown quantization method {m!r}")
        return cls(m, int(d.get("bits", d.get("w_bit", 8))), int(d.get("group_size", d.get("q_group_size", 128))),
                   bool(d.get("desc_act", False)), bool(d.get("sym", True)))


@dataclass
class GptqTensor:
    qweight: torch.Tensor
    qzeros: torch.Tensor
    scales: torch.Tensor
    g_idx: Optional[torch.Tensor] = None
    bias: Optional[torch.Tensor] = None
    bits: int = 4
    group_size: int = 128
    zero_offset: int = 1

    @property
    def shape(self) -> tuple:  # (N, K)
        return (self.qweight.shape[1], self.qweight.shape[0] * 32 // self.bits)

    def dequantize(self) -> torch.Tensor:
        b = self.bits
        per = 32 // b
        mask = (1 << b) - 1
        K = self.qweight.shape[0] * per
        shifts = torch.arange(per, dtype=torch.int32, device=self.qweight.device) * b
        q = ((self.qweight.unsqueeze(1) >> shifts[None, :, None]) & mask).reshape(K, -1)  # [K, N]
        z = ((self.qzeros.unsqueeze(2) >> shifts[None, None, :]) & mask).reshape(self.qzeros.shape[0], -1)
        g = self.g_idx.long() if self.g_idx is not None else \
            torch.arange(K, device=q.device) // self.group_size
        w = self.scales.float()[g] * (q.float() - (z.float()[g] + self.zero_offset))
        return w.T.contiguous()


@dataclass
class AwqTensor:
    qweight: torch.Tensor
    qzeros: torch.Tensor
    scales: torch.Tensor
    bits: int = 4
    group_size: int = 128

    @property
    def shape(self) -> tuple:
        return (self.qweight.shape[1] * 32 // self.bits, self.qweight.shape[0])

    def _unpack_cols(self, packed: torch.Tensor) -> torch.Tensor:
        b = self.bits
        per = 32 // b
        mask = (1 << b) - 1
        shifts = torch.arange(per, dtype=torch.int32, device=packed.device) * b
        vals = (packed.unsqueeze(2) >> shifts[None, None, :]) & mask  # [R, C/8, slot]
        out = torch.empty_like(vals)
        out[:, :, list(AWQ_ORDER)] = vals
        return out.reshape(packed.shape[0], -1)

    def dequantize(self) -> torch.Tensor:
        q = self._unpack_cols(self.qweight)  # [K, N]
        z = self._unpack_cols(self.qzeros)   # [K/g, N]
        g = torch.arange(q.shape[0], device=q.device) // self.group_size
        w = self.scales.float()[g] * (q.float() - z.float()[g])
        return w.T.contiguous()


@dataclass
class Int8Tensor:
    weight: torch.Tensor
    scale: float = 1.0
    zero_point: int = 0

    @property
    def shape(self) -> tuple:
        return tuple(self.weight.shape)

    def dequantize(self) -> torch.Tensor:
        return (self.weight.float() - self.zero_point) * self.scale


def _files(path: str) -> list:
    return sorted(glob.glob(os.path.join(path, "*.safetensors"))) if os.path.isdir(path) else [path]


def _read_all(path: str) -> dict:
    from safetensors.torch import load_file

    out = {}
    for f in _files(path):
        out.update(load_file(f))
    return out


def read_quantization_config(path: str) -> Optional[QuantizationConfig]:
    """``quantize_config.json`` or the ``quantization_config`` entry of ``config.json``."""
    d = path if os.path.isdir(path) else os.path.dirname(path)
    for name in ("quantize_config.json", "quant_config.json"):
        p = os.path.join(d, name)
        if os.path.exists(p):
            with open(p) as f:
                return QuantizationConfig.from_dict(json.load(f))
    p = os.path.join(d, "config.json")
    if os.path.exists(p):
        with open(p) as f:
            qc = json.load(f).get("quantization_config")
        if qc:
            return QuantizationConfig.from_dict(qc)
    return None


def load_gptq(path: str, cfg: Optional[QuantizationConfig] = None, zero_offset: int = 1) -> dict:
    cfg = cfg or read_quantization_config(path) or QuantizationConfig("gptq", 4, 128)
    t = _read_all(path)
    out = {}
    for name in t:
        if name.endswith(".qweight"):
            base = name[:-len(".qweight")]
            if f"{base}.qzeros" in t and f"{base}.scales" in t:
                out[base] = GptqTensor(t[name], t[f"{base}.qzeros"], t[f"{base}.scales"], t.get(f"{base}.g_idx"),
                                       t.get(f"{base}.bias"), cfg.bits, cfg.group_size, zero_offset)
    return out


def load_awq(path: str, cfg: Optional[QuantizationConfig] = None) -> dict:
    cfg = cfg or read_quantization_config(path) or QuantizationConfig("awq", 4, 128)
    t = _read_all(path)
    out = {}
    for name in t:
        if name.endswith(".qweight"):
            base = name[:-len(".qweight")]
            if f"{base}.qzeros" in t and f"{base}.scales" in t:
                out[base] = AwqTensor(t[name], t[f"{base}.qzeros"], t[f"{base}.scales"], cfg.bits, cfg.group_size)
    return out


def load_int8(path: str) -> dict:
    t = _read_all(path)
    out = {}
    for name, w in t.items():
        if name.endswith(".weight") and w.dtype == torch.int8:
            base = name[:-len(".weight")]
            s = t.get(f"{base}.scale")
            z = t.get(f"{base}.zero_point")
            out[base] = Int8Tensor(w, float(s.reshape(-1)[0]) if s is not None else 1.0,
                                   int(z.reshape(-1)[0]) if z is not None else 0)
    return out


def load_quantized(path: str) -> dict:
    """Dispatch on the checkpoint's quantization config (default int8)."""
    cfg = read_quantization_config(path) or QuantizationConfig()
    if cfg.quantization_method == "gptq":
        return load_gptq(path, cfg)
    if cfg.quantization_method == "awq":
        return load_awq(path, cfg)
    return load_int8(path)
