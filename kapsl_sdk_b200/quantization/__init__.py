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

from dataclasses import dataclass

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
