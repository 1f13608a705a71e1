"""Paged KV-cache block bookkeeping, mirroring crates/paraoxidizer-runtime/src/paged_cache.rs.

The reference's BlockManager / BlockTable (paged_cache.rs:69-170) allocate 16-token blocks from
a LIFO free list. Here the same bookkeeping drives the device block tables read by the CUDA
paged decode-attention kernel; the K/V pages themselves live in HBM as f16.
"""
from __future__ import annotations

import numpy as np

DEFAULT_BLOCK_SIZE = 16  # paged_cache.rs:4


class OutOfBlocks(RuntimeError):
    """PoxError::Runtime("PagedAttention Out of Memory ...") (paged_cache.rs:104-110)."""


class BlockManager:
    """paged_cache.rs:69-130: a free list of physical block ids, popped from the end."""

    def __init__(self, total_blocks: int, block_size: int = DEFAULT_BLOCK_SIZE):
        self.block_size = block_size
        self.total_blocks = total_blocks
        self.free_block_ids = list(range(total_blocks))

    def allocate_block(self) -> int:
        if not self.free_block_ids:
            raise OutOfBlocks("PagedAttention Out of Memory: No free physical blocks available")
        return self.free_block_ids.pop()

    def free_block(self, block_id: int) -> None:
        if block_id < self.total_blocks and block_id not in self.free_block_ids:
            self.free_block_ids.append(block_id)

    def available_blocks(self) -> int:
        return len(self.free_block_ids)


class BlockTable:
    """paged_cache.rs:133-170: logical block = pos // block_size, offset = pos % block_size."""

    def __init__(self, block_size: int = DEFAULT_BLOCK_SIZE):
        self.block_size = block_size
        self.allocated_block_ids: list[int] = []
        self.sequence_len = 0

    def append_token(self, manager: BlockManager) -> tuple[int, int]:
        pos = self.sequence_len
        block_idx = pos // self.block_size
        off = pos % self.block_size
        if block_idx >= len(self.allocated_block_ids):
            self.allocated_block_ids.append(manager.allocate_block())
        self.sequence_len += 1
        return self.allocated_block_ids[block_idx], off

    def reserve(self, manager: BlockManager, n_tokens: int) -> None:
        """Allocate blocks up front for n_tokens more tokens (device page tables are fixed-size
        during a captured decode loop)."""
        need = (self.sequence_len + n_tokens + self.block_size - 1) // self.block_size
        while len(self.allocated_block_ids) < need:
            self.allocated_block_ids.append(manager.allocate_block())

    def free(self, manager: BlockManager) -> None:
        for b in self.allocated_block_ids:
            manager.free_block(b)
        self.allocated_block_ids.clear()
        self.sequence_len = 0

    def as_array(self, width: int) -> np.ndarray:
        out = np.full(width, -1, np.int32)
        n = min(width, len(self.allocated_block_ids))
        out[:n] = self.allocated_block_ids[:n]
        return out
