"""Paged KV pool and block allocator with the reference engine's layout.

Mirrors leaninfer/engine/cache_manager.py:
  * BlockAllocator (cache_manager.py:13-42): FIFO free list of block ids
    1..num_blocks-1; block 0 is the trash block that idle CUDA-graph rows
    write into (cache_manager.py:20-25).
  * BlockCache (cache_manager.py:45-76): two bf16 pools
    [num_layers, num_blocks, block_size, num_kv_heads, head_dim]; write()
    scatters k, v [B, Hkv, q_len, D] to block_table[b, col // BS], col % BS,
    col = pos[b] + t. Here write() runs the paged-write kernel instead of
    torch advanced indexing; the result is bit-identical (a copy).
"""
from __future__ import annotations

from collections import deque

import torch

from .flash_attn_interface import paged_kv_write


def blocks_for(n_tokens: int, block_size: int) -> int:
    """Blocks needed to hold n_tokens (ceil division), cache_manager.py:7-9."""
    return -(-n_tokens // block_size)


class InsufficientBlocksError(RuntimeError, AssertionError):
    """allocate(n) with fewer than n free blocks. The reference signals this
    with an assert (cache_manager.py:38, an AssertionError); this error is an
    AssertionError too, so callers catching that keep working, and a
    RuntimeError like the package's other errors. It is raised under -O as
    well, where the reference's assert would vanish."""


class BlockAllocator:
    """FIFO free list of physical block ids; block 0 is reserved as trash."""

    def __init__(self, num_blocks: int) -> None:
        self.free: deque[int] = deque(range(1, num_blocks))

    @property
    def num_free(self) -> int:
        return len(self.free)

    def allocate(self, n: int) -> list[int]:
        if n > len(self.free):
            raise InsufficientBlocksError(f"Insufficient free blocks: asked {n}, free {len(self.free)}")
        return [self.free.popleft() for _ in range(n)]

    def release(self, blocks: list[int]) -> None:
        self.free.extend(blocks)


class BlockCache:
    """K/V pools [L, NB, BS, Hkv, D] bf16 on one device."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 device, dtype=torch.bfloat16, zero: bool = True) -> None:
        shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        alloc = torch.zeros if zero else torch.empty
        self.k = alloc(shape, dtype=dtype, device=device)
        self.v = alloc(shape, dtype=dtype, device=device)
        self.block_size = block_size
        self.device = torch.device(device)

    def write(self, layer: int, block_tables: torch.Tensor, pos: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: [B, Hkv, q_len, D] (the reference layout); pos: [B] int64."""
        kt = k.transpose(1, 2)  # [B, q_len, Hkv, D]
        vt = v.transpose(1, 2)
        n = kt.shape[1]
        if n > 1 and kt.stride(0) != n * kt.stride(1):
            kt = kt.contiguous()
        if n > 1 and vt.stride(0) != n * vt.stride(1):
            vt = vt.contiguous()
        paged_kv_write(kt, vt, pos, block_tables, self.k[layer], self.v[layer])
