"""Paged KV cache: block pool and per-layer cache tensors.

Cache layout per layer: K and V each [num_blocks, kv_heads, block, head_dim]
(one contiguous 16 KB page per (block, head) at head_dim 128), the layout the
attention kernel streams.  Block 0 is reserved as the scratch page that
padded batch rows write into and read from, so a fixed-shape (CUDA-graph)
batch never touches a live request's cache.
"""
from __future__ import annotations

from typing import List

import torch


class BlockPool:
    def __init__(self, num_blocks: int):
        if num_blocks < 2:
            raise ValueError("the KV cache needs at least 2 blocks")
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, 0, -1))  # block 0 reserved

    @property
    def free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> List[int]:
        if n > len(self._free):
            raise MemoryError(f"KV cache exhausted: need {n} blocks, {len(self._free)} free")
        out = self._free[-n:][::-1] if n else []
        del self._free[len(self._free) - n:]
        return out

    def release(self, blocks: List[int]) -> None:
        self._free.extend(reversed(blocks))


def allocate_caches(num_layers: int, shape, dtype, device) -> List[tuple]:
    caches = []
    for _ in range(num_layers):
        k = torch.zeros(shape, dtype=dtype, device=device)
        v = torch.zeros(shape, dtype=dtype, device=device)
        caches.append((k, v))
    return caches


def blocks_for(tokens: int, block_size: int) -> int:
    return (tokens + block_size - 1) // block_size
