"""GPU paged KV pool.

One allocation holds every layer's K and V pages:
``[layers, 2, num_blocks, kv_heads, block_size, head_dim]`` (bf16).  A page
(block, kv head) is a contiguous 4 KiB run for head_dim 128, which is what the
TMA-fed attention kernels load.  The reference keeps f16 pages in host RAM
(crates/kapsl-llm/src/kv_cache.rs:823-1796) and copies them to the device
every step; here the pages never leave HBM, and only block ids move.

Also: CPU offload of whole sequences into pinned host memory (reference
``CpuKvBlockStore``, kv_cache.rs:724-821, 940-1084).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class KVLayout:
    num_layers: int
    num_kv_heads: int
    head_dim: int
    block_size: int = 16
    dtype: torch.dtype = torch.bfloat16

    def bytes_per_block(self) -> int:
        return self.num_layers * 2 * self.num_kv_heads * self.block_size * self.head_dim * \
            torch.tensor([], dtype=self.dtype).element_size()


class KVPool:
    def __init__(self, layout: KVLayout, num_blocks: int, device, shareable: bool = False):
        """``shareable``: allocate the pages with cudaMalloc so that another process
        (the prefill side of a disaggregated deployment) can map them with CUDA IPC
        and write KV blocks into them directly."""
        self.layout = layout
        self.num_blocks = num_blocks
        self.device = torch.device(device)
        L = layout
        shape = (L.num_layers, 2, num_blocks, L.num_kv_heads, L.block_size, L.head_dim)
        self._raw = 0
        if shareable and self.device.type == "cuda":
            from .._ext import cuda_ops

            c = cuda_ops()
            nbytes = L.bytes_per_block() * num_blocks
            with torch.cuda.device(self.device):
                self._raw = c.symm_alloc(nbytes)  # zero-filled
                self.storage = c.tensor_from_ptr(self._raw, list(shape), "bfloat16", self.device.index)
        else:
            self.storage = torch.zeros(shape, dtype=L.dtype, device=self.device)
        self._in_flight: list = []  # (event, pinned host copy) read by a queued restore
        self.k = [self.storage[i, 0] for i in range(L.num_layers)]
        self.v = [self.storage[i, 1] for i in range(L.num_layers)]

    def ipc_handle(self) -> str:
        """CUDA IPC handle of a shareable pool (see ``shareable``)."""
        if not self._raw:
            raise RuntimeError("KV pool was not allocated shareable")
        from .._ext import cuda_ops

        return cuda_ops().symm_handle(self._raw)

    def close(self) -> None:
        if self._raw:
            from .._ext import cuda_ops

            torch.cuda.synchronize(self.device)
            self.storage = None
            cuda_ops().symm_free(self._raw)
            self._raw = 0

    @staticmethod
    def blocks_for_bytes(layout: KVLayout, nbytes: int) -> int:
        return max(1, nbytes // layout.bytes_per_block())

    @property
    def nbytes(self) -> int:
        return self.storage.numel() * self.storage.element_size()

    # ------------------------------------------------------------ offload
    def offload(self, blocks: list[int]) -> torch.Tensor:
        """Copy pages of ``blocks`` (all layers) into host memory (pinned on a GPU
        pool: one kernel writes them straight into it over unified addressing)."""
        L = self.layout
        host = torch.empty((L.num_layers, 2, len(blocks)) + tuple(self.storage.shape[3:]),
                           dtype=self.storage.dtype, pin_memory=self.device.type == "cuda")
        if self.device.type == "cuda" and blocks:
            src = torch.as_tensor(blocks, dtype=torch.int32).to(self.device, non_blocking=True)
            dst = torch.arange(len(blocks), dtype=torch.int32, device=self.device)
            self._copy(self.storage.data_ptr(), host.data_ptr(), src, dst, self.num_blocks, len(blocks))
        elif blocks:
            host.copy_(self.storage.index_select(2, torch.as_tensor(blocks, dtype=torch.long)))
        return host

    def restore(self, host: torch.Tensor, blocks: list[int]) -> None:
        """Copy offloaded pages back into (possibly different) ``blocks``."""
        if self.device.type == "cuda" and blocks:
            src = torch.arange(len(blocks), dtype=torch.int32, device=self.device)
            dst = torch.as_tensor(blocks, dtype=torch.int32).to(self.device, non_blocking=True)
            self._copy(host.data_ptr(), self.storage.data_ptr(), src, dst, len(blocks), self.num_blocks)
            # the kernel reads ``host`` later on the stream: keep it until then
            ev = torch.cuda.Event()
            ev.record()
            self._in_flight.append((ev, host))
        elif blocks:
            self.storage.index_copy_(2, torch.as_tensor(blocks, dtype=torch.long), host)
        self._in_flight = [(e, h) for e, h in self._in_flight if not e.query()]

    def _copy(self, src_ptr: int, dst_ptr: int, src_ids, dst_ids, src_blocks: int, dst_blocks: int) -> None:
        from .._ext import cuda_ops

        L = self.layout
        cuda_ops().kv_copy_blocks(src_ptr, dst_ptr, src_ids, dst_ids, L.num_layers * 2, src_blocks, dst_blocks,
                                  L.bytes_per_block() // (L.num_layers * 2))

    def copy_blocks(self, src: list[int], dst: list[int]) -> None:
        """Duplicate pages (copy-on-write of a shared prefix block)."""
        s = torch.as_tensor(src, dtype=torch.long, device=self.device)
        d = torch.as_tensor(dst, dtype=torch.long, device=self.device)
        self.storage.index_copy_(2, d, self.storage.index_select(2, s))
