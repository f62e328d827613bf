"""Quantized weights.

* :class:`QuantWeight` — a linear layer's weight kept in a block-quantized
  format on the GPU; :func:`kapsl_sdk_b200.ops.linear` dispatches it to the
  matching fused kernel (GGUF Q4_K: dequantized into tensor memory inside the
  tcgen05 GEMM mainloop, csrc/cuda/gemm_q4k.cu).
* :func:`quantize_q4_k` / :func:`dequantize_q4_k` — GPU quantizer (same
  rounding steps as :func:`kapsl_sdk_b200.loaders.gguf.quantize_q4_k`) and
  dequantizer.
* :mod:`.safetensors_loaders` — GPTQ / AWQ / INT8 checkpoint readers with the
  dequantization math.

Reference counterpart: crates/kapsl-quantization (config.rs:3-30,
tensor.rs:4-35, loader/*.rs) parses GPTQ/AWQ/INT8 tensors but has no dequant
math and is not used by any model path; GGUF k-quants are served there by
llama.cpp (crates/kapsl-llm/src/gguf_backend.rs:110-118).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch

Q4_K_BLOCK = 256
Q4_K_BYTES = 144


@dataclass
class QuantWeight:
    """Weight [n, k] stored as packed quantized blocks (uint8, n * bytes_per_row bytes).

    ``tiled``: the Q4_K blocks are reordered tile-major, [n/128][k/256][128 rows][144 B],
    so each 128-row tile's super-block is one contiguous 18 KiB copy for the GEMM
    (the row-major GGUF order needs one strided 144-byte piece per row)."""
    raw: torch.Tensor
    n: int
    k: int
    fmt: str = "q4_k"
    tiled: bool = False

    @property
    def shape(self) -> tuple:
        return (self.n, self.k)

    @property
    def device(self) -> torch.device:
        return self.raw.device

    def nbytes(self) -> int:
        return self.raw.numel()

    def row_major(self) -> torch.Tensor:
        """The blocks in GGUF row order (uint8 [n, k/256 * 144])."""
        if not self.tiled:
            return self.raw
        nsb = self.k // Q4_K_BLOCK
        return self.raw.view(self.n // 128, nsb, 128, Q4_K_BYTES).permute(0, 2, 1, 3).reshape(self.n, -1)

    def dequantize(self) -> torch.Tensor:
        return dequantize_q4_k(self.row_major().contiguous(), self.n, self.k)


def tile_q4_k(raw: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """Row-major Q4_K blocks [n, k/256 * 144] -> tile-major order (n % 128 == 0)."""
    nsb = k // Q4_K_BLOCK
    return raw.view(n // 128, 128, nsb, Q4_K_BYTES).permute(0, 2, 1, 3).contiguous().view(n, nsb * Q4_K_BYTES)


def from_gguf_blocks(raw: torch.Tensor, n: int, k: int, tiled: bool = True) -> QuantWeight:
    """Wrap GGUF Q4_K bytes (row-major, as stored in the file) for the fused GEMM."""
    raw = raw.reshape(n, k // Q4_K_BLOCK * Q4_K_BYTES)
    if tiled and n % 128 == 0:
        return QuantWeight(tile_q4_k(raw, n, k), n, k, "q4_k", True)
    return QuantWeight(raw.contiguous(), n, k, "q4_k", False)


def quantize_q4_k(w: torch.Tensor, tiled: bool = True) -> QuantWeight:
    """bf16 [n, k] (k % 256 == 0) on the GPU -> Q4_K QuantWeight (tile-major
    when ``tiled`` and n % 128 == 0)."""
    from .._ext import cuda_ops

    n, k = w.shape
    if k % Q4_K_BLOCK:
        raise ValueError(f"Q4_K needs the input dimension to be a multiple of 256 (got {k})")
    w = w.to(torch.bfloat16).contiguous()
    raw = torch.empty(n, k // Q4_K_BLOCK * Q4_K_BYTES, dtype=torch.uint8, device=w.device)
    cuda_ops().q4k_quantize(w, raw)
    return from_gguf_blocks(raw, n, k, tiled)


def dequantize_q4_k(raw: torch.Tensor, n: int, k: int) -> torch.Tensor:
    from .._ext import cuda_ops

    out = torch.empty(n, k, dtype=torch.bfloat16, device=raw.device)
    cuda_ops().q4k_dequant(raw.contiguous(), out)
    return out


class PackedRows:
    """GGUF k-quant weight rows kept packed for the CPU backend: ``raw`` is
    uint8 [N, K / 256 * BLOCK] (one row per output feature).  Short activations
    (decode) go through the native kernels on the packed blocks; long ones
    dequantize row blocks into a BLAS matmul.  Subclasses name the format."""

    FMT = ""
    BLOCK = 0
    INT8_KERNEL = FP32_KERNEL = DEQUANT = ""

    def __init__(self, raw, k: int):
        import numpy as np

        self.raw = np.ascontiguousarray(raw, dtype=np.uint8)
        self.k = int(k)
        if self.raw.ndim != 2 or self.k % 256 or self.raw.shape[1] != self.k // 256 * self.BLOCK:
            raise ValueError(f"{self.FMT} rows: raw must be [N, K / 256 * {self.BLOCK}] with K a multiple of 256")

    @property
    def n(self) -> int:
        return self.raw.shape[0]

    @property
    def shape(self) -> tuple:
        return (self.n, self.k)

    def rows(self, a: int, b: int) -> "PackedRows":
        return type(self)(self.raw[a:b], self.k)

    def take(self, idx) -> "PackedRows":
        return type(self)(self.raw[idx], self.k)

    @staticmethod
    def cat(parts: list) -> "PackedRows":
        import numpy as np

        return type(parts[0])(np.concatenate([p.raw for p in parts], 0), parts[0].k)

    def dequantize(self) -> torch.Tensor:
        from .._ext import native

        out = torch.empty(self.n, self.k, dtype=torch.float32)
        getattr(native().cpu, self.DEQUANT)(self.raw, 0, self.n, out.numpy())
        return out

    def matmul(self, x: torch.Tensor, row_block: int = 2048, int8: Optional[bool] = None) -> torch.Tensor:
        """x [T, K] fp32 -> x @ W.T [T, N].

        Up to 16 rows (decode) run the native kernels on the packed blocks:
        with ``int8`` (default unless ``KAPSL_CPU_Q4K_INT8=0``) the activations
        are rounded to int8 per 256-value block and multiplied with the quants
        in integer arithmetic (llama.cpp's k-quant x Q8_K scheme; under 1% of
        the output range), otherwise each block is dequantized to fp32 first.
        More rows dequantize ``row_block`` weight rows at a time into one fp32
        buffer and use BLAS."""
        from .._ext import native

        cpu = native().cpu
        x = x.float().contiguous()
        y = torch.empty(x.shape[0], self.n, dtype=torch.float32)
        if x.shape[0] <= 16:
            if int8 is None:
                int8 = os.environ.get("KAPSL_CPU_Q4K_INT8", "1") != "0"
            kernel = self.INT8_KERNEL if int8 or not self.FP32_KERNEL else self.FP32_KERNEL
            getattr(cpu, kernel)(x.numpy(), self.raw, y.numpy())
            return y
        buf = torch.empty(min(row_block, self.n), self.k, dtype=torch.float32)
        deq = getattr(cpu, self.DEQUANT)
        for n0 in range(0, self.n, row_block):
            n1 = min(self.n, n0 + row_block)
            w = buf[:n1 - n0]
            deq(self.raw, n0, n1, w.numpy())
            y[:, n0:n1] = x @ w.T
        return y


class Q4KRows(PackedRows):
    """Q4_K rows (144-byte blocks): int8-activation and fp32-activation decode kernels."""

    FMT, BLOCK = "Q4_K", 144
    INT8_KERNEL, FP32_KERNEL, DEQUANT = "q4k_matmul_q8", "q4k_matmul", "q4k_dequant_rows"


class Q6KRows(PackedRows):
    """Q6_K rows (210-byte blocks; the output and some FFN-down / V weights of
    Q4_K_M files): int8-activation decode kernel."""

    FMT, BLOCK = "Q6_K", 210
    INT8_KERNEL, FP32_KERNEL, DEQUANT = "q6k_matmul_q8", "", "q6k_dequant_rows"


class Q80Rows(PackedRows):
    """Q8_0 rows (34-byte blocks of 32 values; K a multiple of 256): int8-activation decode kernel."""

    FMT, BLOCK = "Q8_0", 272  # bytes per 256 values (8 blocks of 34)
    INT8_KERNEL, FP32_KERNEL, DEQUANT = "q80_matmul_q8", "", "q80_dequant_rows"


class RowStack:
    """Row-concatenation of weights of different formats (packed rows of two
    k-quant types, or packed and fp32 rows): each part multiplies on its own
    and the outputs are joined."""

    def __init__(self, parts: list):
        self.parts = list(parts)
        self.k = int(self.parts[0].shape[1])
        self.n = sum(int(p.shape[0]) for p in self.parts)

    @property
    def shape(self) -> tuple:
        return (self.n, self.k)

    def matmul(self, x: torch.Tensor) -> torch.Tensor:
        return torch.cat([p.matmul(x) if isinstance(p, PackedRows) else x @ p.T for p in self.parts], 1)

    def dequantize(self) -> torch.Tensor:
        return torch.cat([p.dequantize() if isinstance(p, PackedRows) else p for p in self.parts], 0)
