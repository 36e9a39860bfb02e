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

The reference is single-GPU (it uses no torch.distributed at all); these
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


class _CudaBuffer:
    """A device pointer exposed through __cuda_array_interface__ (int16 words)."""

    def __init__(self, ptr: int, n_words: int):
        self.__cuda_array_interface__ = {"shape": (n_words,), "typestr": "<i2", "data": (ptr, False), "version": 3,
                                         "strides": None}


class NVLinkAllGatherDecode:
    """KV-head-sharded decode with the all-gather fused into the decode
    kernels: every rank's decode/combine kernels store its heads' outputs
    straight into every rank's gather buffer over NVLink (CUDA IPC peer
    mappings); a one-warp device barrier on the same stream (publish this
    rank's epoch, wait bounded for the peers') makes the gathered
    [B, 1, Hq, D] output safe to read. No NCCL call and no copy kernel.

    The gather buffer has `slots` slots used in turn (slot = call index mod
    slots, chosen by the caller, e.g. layer index mod 2): a peer may already
    be writing call n+1 while this rank still reads call n.
    """

    SIG_BYTES = 256

    def __init__(self, shard: HeadShard, max_batch: int, group=None, slots: int = 2, head_dim: int = 128):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self._ct = ctypes
        self._lib = _lib
        self.shard, self.group, self.slots = shard, group, slots
        self.P, self.rank = shard.world, shard.rank
        self.hq_total = shard.num_q_heads * shard.world
        self.D = head_dim
        self.max_batch = max_batch
        slot_elems = max_batch * self.hq_total * head_dim
        self.slot_bytes = (slot_elems * 2 + 255) // 256 * 256
        nbytes = self.SIG_BYTES + slots * self.slot_bytes
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        _lib.call("la_p2p_alloc", nbytes, ctypes.byref(ptr), handle)
        self._own = ptr
        handles = [None] * self.P
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        bases = []
        for r in range(self.P):
            if r == self.rank:
                bases.append(ptr.value)
            else:
                pp = ctypes.c_void_p()
                _lib.call("la_p2p_open", ctypes.create_string_buffer(handles[r], 64), ctypes.byref(pp))
                self._opened.append(pp)
                bases.append(pp.value)
        self._bases = bases
        self._signals = (ctypes.c_void_p * self.P)(*bases)
        self._slot_ptrs = [(ctypes.c_void_p * self.P)(*[b + self.SIG_BYTES + s * self.slot_bytes for b in bases])
                           for s in range(slots)]
        words = torch.as_tensor(_CudaBuffer(ptr.value + self.SIG_BYTES, slots * self.slot_bytes // 2),
                                device=torch.device("cuda", torch.cuda.current_device()))
        per = self.slot_bytes // 2
        self.local = [words[s * per: s * per + slot_elems].view(torch.bfloat16).view(max_batch, self.hq_total, head_dim)
                      for s in range(slots)]
        self._ws = None

    def __call__(self, q_local: torch.Tensor, k_cache_local: torch.Tensor, v_cache_local: torch.Tensor,
                 cache_seqlens: torch.Tensor, block_table: torch.Tensor, slot: int = 0,
                 softmax_scale: Optional[float] = None, wait: bool = True) -> torch.Tensor:
        """q_local [B, 1, Hq/P, D] -> gathered [B, 1, Hq, D] (a view of this
        rank's gather slot, valid until the slot is reused). With wait=False
        the call only publishes this rank's epoch: the slot may still be
        filling, and the next kernel on the stream must wait for each peer
        itself (o_proj does)."""
        from . import flash_attn_interface as fai

        ct, lib = self._ct, self._lib
        B, _, hq, D = q_local.shape
        if B > self.max_batch or hq != self.shard.num_q_heads or D != self.D:
            raise RuntimeError("q_local does not match the gather buffer")
        dev = q_local.device.index
        fai.ensure_init(dev)
        need = fai.decode_workspace_bytes(dev, hq, k_cache_local.shape[2], D)
        ws = fai._workspace(dev, need)
        err = fai.error_word(dev)
        stream = ct.c_void_p(torch.cuda.current_stream(q_local.device).cuda_stream)
        scale = D ** -0.5 if softmax_scale is None else float(softmax_scale)
        kc = k_cache_local
        lib.call("la_paged_decode_allgather",
                 ct.c_void_p(q_local.data_ptr()), q_local.stride(0), q_local.stride(2),
                 ct.c_void_p(kc.data_ptr()), ct.c_void_p(v_cache_local.data_ptr()),
                 kc.stride(0), kc.stride(1), kc.stride(2), kc.shape[0], kc.shape[1],
                 ct.c_void_p(block_table.data_ptr()), block_table.stride(0), block_table.shape[1],
                 ct.c_void_p(cache_seqlens.data_ptr()),
                 B, hq, kc.shape[2], D, ct.c_float(scale),
                 self._slot_ptrs[slot], self.hq_total * D, D,
                 self.rank, self.P,
                 ct.c_void_p(ws.data_ptr()), ws.numel(),
                 ct.c_void_p(err.data_ptr()), stream)
        lib.call("la_p2p_barrier" if wait else "la_p2p_publish", self._signals, self.P, self.rank,
                 ct.c_void_p(err.data_ptr()), stream)
        return self.local[slot][:B].view(B, 1, self.hq_total, D)

    def o_proj(self, gathered: torch.Tensor, weight: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """o_proj (model.py:68-69) of a gathered slot on the tcgen05 GEMM that
        waits for each peer's heads as they land (la_o_proj_gathered):
        gathered [B, 1, Hq, D] from __call__(..., wait=False), weight
        [hidden, Hq*D] bf16 -> [B, hidden] bf16, the same on every rank."""
        from . import flash_attn_interface as fai

        ct, lib = self._ct, self._lib
        B = gathered.shape[0]
        K = self.hq_total * self.D
        if weight.dim() != 2 or weight.shape[1] != K or weight.dtype != torch.bfloat16 or weight.stride(1) != 1:
            raise RuntimeError("weight must be bf16 [hidden, Hq*D] with a contiguous last axis")
        a = gathered.view(B, K)
        N = weight.shape[0]
        if out is None:
            out = torch.empty(B, N, dtype=torch.bfloat16, device=gathered.device)
        dev = gathered.device.index
        fai.ensure_init(dev)
        stream = ct.c_void_p(torch.cuda.current_stream(gathered.device).cuda_stream)
        lib.call("la_o_proj_gathered", ct.c_void_p(a.data_ptr()), a.stride(0), ct.c_void_p(weight.data_ptr()),
                 weight.stride(0), ct.c_void_p(out.data_ptr()), out.stride(0), B, N, K,
                 ct.c_void_p(self._bases[self.rank]), self.P, self.rank,
                 ct.c_void_p(fai.error_word(dev).data_ptr()), stream)
        return out

    def attention_o_proj(self, q_local: torch.Tensor, k_cache_local: torch.Tensor, v_cache_local: torch.Tensor,
                         cache_seqlens: torch.Tensor, block_table: torch.Tensor, o_proj_weight: torch.Tensor,
                         slot: int = 0, softmax_scale: Optional[float] = None) -> torch.Tensor:
        """One KV-head-sharded attention layer up to o_proj's output: decode on
        this rank's heads with the all-gather stores fused in, an epoch
        publish, and the o_proj GEMM consuming the peers' heads as they land.
        Returns [B, hidden] (identical on every rank)."""
        g = self(q_local, k_cache_local, v_cache_local, cache_seqlens, block_table, slot=slot,
                 softmax_scale=softmax_scale, wait=False)
        return self.o_proj(g, o_proj_weight)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective)."""
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for pp in self._opened:
            self._lib.call("la_p2p_close", pp)
        self._opened = []
        dist.barrier(group=self.group)
        self.local = []
        if self._own is not None:
            self._lib.call("la_p2p_free", self._own)
            self._own = None
