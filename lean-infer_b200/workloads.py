"""Seeded synthetic inputs with the shapes and distributions of the
benchmark configurations (Qwen3-0.6B attention shapes: 16 query heads over
8 kv heads, head_dim 128, 256-token blocks).

decode_batch   a paged decode step: per-sequence context lengths uniform in
               [ctx_lo, ctx_hi], block tables dealt from a seeded random
               permutation of the block ids 1..NB-1 (block 0 = trash block),
               q and the pool N(0,1).
prefill_batch  packed causal prefill: prompt lengths uniform in [lo, hi],
               cu_seqlens from them, blocks from a seeded shuffled free list.

Generation happens on the requested device with a seeded generator, so large
pools are made in place instead of on the host.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class DecodeBatch:
    q: torch.Tensor             # [B, 1, Hq, D] bf16
    k_cache: torch.Tensor       # [NB, BS, Hkv, D] bf16
    v_cache: torch.Tensor
    block_table: torch.Tensor   # [B, max_blocks] int32
    cache_seqlens: torch.Tensor  # [B] int32

    @property
    def kv_bytes(self) -> int:
        """Algorithmic K+V bytes one decode pass reads."""
        return int(self.cache_seqlens.clamp(min=0).sum()) * self.k_cache.shape[2] * self.k_cache.shape[3] * 2 * 2


def seq_lengths(batch: int, lo: int, hi: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (batch,), generator=g, dtype=torch.int64)


def deal_blocks(lengths: torch.Tensor, block_size: int, num_blocks: int | None, seed: int):
    """Block tables from a seeded random permutation of 1..NB-1. If
    num_blocks is None it is sized to fit every sequence (+ the trash block)."""
    need = [(-(-int(n) // block_size)) for n in lengths]
    total = sum(need)
    if num_blocks is None:
        num_blocks = total + 1
    if total > num_blocks - 1:
        raise ValueError(f"{total} blocks needed, pool has {num_blocks - 1} usable")
    g = torch.Generator().manual_seed(seed + 7919)
    perm = (torch.randperm(num_blocks - 1, generator=g) + 1).to(torch.int32)
    max_blocks = max(need) if need else 1
    bt = torch.zeros(len(need), max(max_blocks, 1), dtype=torch.int32)
    o = 0
    for b, n in enumerate(need):
        bt[b, :n] = perm[o:o + n]
        o += n
    return bt, num_blocks


def decode_batch(batch: int, ctx_lo: int, ctx_hi: int, *, num_blocks: int | None = 512, block_size: int = 256,
                 num_q_heads: int = 16, num_kv_heads: int = 8, head_dim: int = 128, seed: int = 0,
                 device="cpu", lengths: torch.Tensor | None = None) -> DecodeBatch:
    dev = torch.device(device)
    if lengths is None:
        lengths = seq_lengths(batch, ctx_lo, ctx_hi, seed)
    bt, nb = deal_blocks(lengths, block_size, num_blocks, seed)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    kc = _randn_bf16((nb, block_size, num_kv_heads, head_dim), g, dev)
    vc = _randn_bf16((nb, block_size, num_kv_heads, head_dim), g, dev)
    q = torch.randn((batch, 1, num_q_heads, head_dim), generator=g, device=dev).to(torch.bfloat16)
    return DecodeBatch(q, kc, vc, bt.to(dev), lengths.to(torch.int32).to(dev))


def _randn_bf16(shape, g, dev):
    out = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    flat = out.view(-1)
    step = 1 << 28
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n] = torch.randn(n, generator=g, device=dev)
    return out


@dataclass
class PrefillBatch:
    q: torch.Tensor           # [T, Hq, D] bf16
    k: torch.Tensor           # [T, Hkv, D]
    v: torch.Tensor
    cu_seqlens: torch.Tensor  # [B+1] int32
    lengths: torch.Tensor     # [B] int64
    block_table: torch.Tensor
    num_blocks: int

    @property
    def causal_flops(self) -> float:
        """4 * Hq * D * sum(L^2) / 2 (QK^T and PV, causal half)."""
        Hq, D = self.q.shape[1], self.q.shape[2]
        return float(2 * Hq * D * (self.lengths.double() ** 2).sum())


def prefill_batch(batch: int, lo: int, hi: int, *, block_size: int = 256, num_q_heads: int = 16,
                  num_kv_heads: int = 8, head_dim: int = 128, seed: int = 0, device="cpu",
                  lengths: torch.Tensor | None = None) -> PrefillBatch:
    dev = torch.device(device)
    if lengths is None:
        lengths = seq_lengths(batch, lo, hi, seed)
    cu = torch.zeros(batch + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lengths, 0).to(torch.int32)
    T = int(cu[-1])
    bt, nb = deal_blocks(lengths, block_size, None, seed)
    g = torch.Generator(device=dev).manual_seed(seed + 2)
    q = torch.randn((T, num_q_heads, head_dim), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((T, num_kv_heads, head_dim), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((T, num_kv_heads, head_dim), generator=g, device=dev).to(torch.bfloat16)
    return PrefillBatch(q, k, v, cu.to(dev), lengths, bt.to(dev), nb)


@dataclass
class ChunkBatch:
    q: torch.Tensor              # [B, chunk, Hq, D] bf16
    k_cache: torch.Tensor        # [NB, BS, Hkv, D] bf16 (prefix + chunk keys written)
    v_cache: torch.Tensor
    block_table: torch.Tensor    # [B, max_blocks] int32
    cache_seqlens: torch.Tensor  # [B] int32: prefix + chunk

    @property
    def causal_flops(self) -> float:
        """4 * Hq * D * sum over queries of the keys each sees (bottom-right
        causal: query i of n sees K - n + i + 1 keys)."""
        B, n, Hq, D = self.q.shape
        K = self.cache_seqlens.double().cpu()
        seen = (K - n) * n + n * (n + 1) / 2
        return float(4 * Hq * D * seen.sum())


def chunk_batch(batch: int, chunk: int, prefix_lo: int, prefix_hi: int, *, block_size: int = 256,
                num_q_heads: int = 16, num_kv_heads: int = 8, head_dim: int = 128, seed: int = 0,
                device="cpu") -> ChunkBatch:
    """Chunked prefill step: every sequence has a prefix of U[prefix_lo,
    prefix_hi] tokens already cached and a `chunk`-token chunk whose keys are
    written too (cache_seqlens = prefix + chunk)."""
    dev = torch.device(device)
    k_lens = seq_lengths(batch, prefix_lo, prefix_hi, seed) + chunk
    bt, nb = deal_blocks(k_lens, block_size, None, seed)
    g = torch.Generator(device=dev).manual_seed(seed + 3)
    kc = _randn_bf16((nb, block_size, num_kv_heads, head_dim), g, dev)
    vc = _randn_bf16((nb, block_size, num_kv_heads, head_dim), g, dev)
    q = torch.randn((batch, chunk, num_q_heads, head_dim), generator=g, device=dev).to(torch.bfloat16)
    return ChunkBatch(q, kc, vc, bt.to(dev), k_lens.to(torch.int32).to(dev))
