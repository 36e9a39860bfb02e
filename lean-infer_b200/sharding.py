"""Multi-GPU partitionings of decode attention (one process per GPU).

request sharding   rank r serves its own slice of the requests with its own
                   pool, allocator and block tables; no collective touches the
                   data path (the benchmark's default, weak scaling).

KV-head sharding   rank r of P holds kv heads [r*Hkv/P, (r+1)*Hkv/P) of every
                   request and the G = Hq/Hkv query heads of each (the mapping
                   q_head // G = kv_head of model.py:57 / flash-attn GQA), in a
                   pool [NB, BS, Hkv/P, D]. Each rank runs the decode kernel on
                   its heads; the [B, Hq/P, D] outputs are all-gathered over
                   NCCL (NVLink/NVSwitch) into [B, Hq, D] before o_proj.

The reference is single-GPU (SURVEY: no torch.distributed anywhere); these
are the two partitionings its decode step admits.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_lo: int
    kv_hi: int
    q_lo: int
    q_hi: int

    @property
    def num_kv_heads(self) -> int:
        return self.kv_hi - self.kv_lo

    @property
    def num_q_heads(self) -> int:
        return self.q_hi - self.q_lo


def kv_head_shard(rank: int, world: int, num_kv_heads: int = 8, num_q_heads: int = 16) -> HeadShard:
    """Rank r's contiguous block of kv heads and the query heads that read them."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    if num_q_heads % num_kv_heads:
        raise ValueError("num_q_heads must be a multiple of num_kv_heads")
    per = num_kv_heads // world
    g = num_q_heads // num_kv_heads
    lo = rank * per
    return HeadShard(rank, world, lo, lo + per, lo * g, (lo + per) * g)


def request_shard(rank: int, world: int, num_requests: int) -> range:
    """Contiguous, near-equal slice of the request ids for rank r."""
    base, extra = divmod(num_requests, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


class KVHeadShardedDecode:
    """Decode attention over a KV-head-sharded pool, gathered over a process
    group. `local_attn(q_local, k_local, v_local, cache_seqlens, block_table)`
    computes this rank's heads ([B, 1, Hq/P, D]); by default it is the sm_100a
    paged decode kernel (flash_attn_with_kvcache)."""

    def __init__(self, shard: HeadShard, group=None, local_attn: Optional[Callable] = None):
        import torch.distributed as dist

        self.dist = dist
        self.shard = shard
        self.group = group
        if local_attn is None:
            from .flash_attn_interface import flash_attn_with_kvcache

            def local_attn(q, kc, vc, seqlens, bt):
                return flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seqlens, block_table=bt, causal=True)

        self.local_attn = local_attn
        self._gather_buf: Optional[torch.Tensor] = None

    def __call__(self, q_local: torch.Tensor, k_cache_local: torch.Tensor, v_cache_local: torch.Tensor,
                 cache_seqlens: torch.Tensor, block_table: torch.Tensor) -> torch.Tensor:
        """q_local [B, 1, Hq/P, D] -> gathered attention output [B, 1, Hq, D]."""
        o = self.local_attn(q_local, k_cache_local, v_cache_local, cache_seqlens, block_table)
        return self.gather(o)

    def gather(self, o_local: torch.Tensor) -> torch.Tensor:
        """[B, 1, Hq/P, D] on every rank -> [B, 1, Hq, D] with the heads in
        rank order (rank r's block of query heads at [q_lo, q_hi))."""
        P = self.shard.world
        B, one, hq_local, D = o_local.shape
        src = o_local.contiguous().view(-1)
        n = src.numel()
        if self._gather_buf is None or self._gather_buf.numel() != n * P or self._gather_buf.device != src.device \
                or self._gather_buf.dtype != src.dtype:
            self._gather_buf = torch.empty(n * P, dtype=src.dtype, device=src.device)
        self.dist.all_gather_into_tensor(self._gather_buf, src, group=self.group)
        # [P, B, 1, Hq/P, D] -> [B, 1, P, Hq/P, D]
        return self._gather_buf.view(P, B, one, hq_local, D).permute(1, 2, 0, 3, 4).reshape(B, one, P * hq_local, D)


def shard_pool(k_cache: torch.Tensor, v_cache: torch.Tensor, shard: HeadShard):
    """This rank's slice [NB, BS, Hkv/P, D] of a full [NB, BS, Hkv, D] pool
    (contiguous copies, as a rank would hold them)."""
    return (k_cache[:, :, shard.kv_lo:shard.kv_hi].contiguous(),
            v_cache[:, :, shard.kv_lo:shard.kv_hi].contiguous())
