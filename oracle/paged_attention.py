"""Oracle for kernels (b) and (c): paged decode and causal varlen prefill
attention in fp32 on the CPU.

Test infrastructure only (see oracle/__init__.py).

Decode follows the contract of flash_attn_with_kvcache as the reference calls
it (leaninfer/qwen3/model.py:58-67): row b's query attends to keys
0..cache_seqlens[b]-1 of kv head h // (Hq/Hkv), key t being
k_cache[block_table[b, t // BS], t % BS] (gather-on-read through the block
table, as the commented SlotCache.read at cache_manager.py:109-118 does for
slots). With one query token, causal (bottom-right aligned) masking removes
nothing. A row with no keys yields zeros (flash-attn returns zeros for fully
masked rows). The attention itself is torch's fp32
F.scaled_dot_product_attention with enable_gqa=True — the reference's CPU
path (model.py:56-57).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def gather_kv(k_layer: torch.Tensor, v_layer: torch.Tensor, bt_row: torch.Tensor, ctx: int):
    """Keys/values 0..ctx-1 of one sequence, [ctx, Hkv, D]."""
    bs = k_layer.shape[1]
    nblk = -(-ctx // bs)
    idx = bt_row[:nblk].long()
    k = k_layer[idx].reshape(-1, *k_layer.shape[2:])[:ctx]
    v = v_layer[idx].reshape(-1, *v_layer.shape[2:])[:ctx]
    return k, v


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                 cache_seqlens: torch.Tensor, softmax_scale: float | None = None, return_lse: bool = False):
    """q: [B, 1, Hq, D]; k/v_cache: [NB, BS, Hkv, D]. Returns fp32 out
    [B, 1, Hq, D] (and natural-log lse [B, Hq])."""
    B, _, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else softmax_scale
    out = torch.zeros(B, 1, Hq, D, dtype=torch.float32)
    lse = torch.full((B, Hq), float("-inf"), dtype=torch.float32)
    for b in range(B):
        ctx = int(cache_seqlens[b])
        if ctx <= 0:
            continue
        k, v = gather_kv(k_cache, v_cache, block_table[b], ctx)
        qb = q[b, 0].float()[None, :, None, :]  # [1, Hq, 1, D]
        kb = k.float().permute(1, 0, 2)[None]   # [1, Hkv, ctx, D]
        vb = v.float().permute(1, 0, 2)[None]
        o = F.scaled_dot_product_attention(qb, kb, vb, scale=scale, enable_gqa=True)
        out[b, 0] = o[0, :, 0]
        if return_lse:
            kr = kb[0].repeat_interleave(Hq // Hkv, dim=0)  # [Hq, ctx, D]
            s = torch.einsum("hd,htd->ht", qb[0, :, 0], kr) * scale
            lse[b] = torch.logsumexp(s, dim=-1)
    return (out, lse) if return_lse else out


def paged_decode_padded(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                        cache_seqlens: torch.Tensor, softmax_scale: float | None = None):
    """The same decode math batched: gather every row's keys into a padded
    [B, Hkv, maxctx, D] fp32 tensor and run one masked SDPA. Used as the timed
    CPU baseline (one SDPA call per layer instead of B)."""
    B, _, Hq, D = q.shape
    bs = k_cache.shape[1]
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else softmax_scale
    ctx = cache_seqlens.long().clamp(min=0)
    maxctx = int(ctx.max()) if B else 0
    nblk = -(-maxctx // bs)
    idx = block_table[:, :nblk].long()  # [B, nblk]
    k = k_cache[idx].reshape(B, nblk * bs, *k_cache.shape[2:])[:, :maxctx].float().transpose(1, 2)
    v = v_cache[idx].reshape(B, nblk * bs, *v_cache.shape[2:])[:, :maxctx].float().transpose(1, 2)
    mask = (torch.arange(maxctx)[None, :] < ctx[:, None])[:, None, None, :]  # [B,1,1,maxctx]
    o = F.scaled_dot_product_attention(q.float().transpose(1, 2), k, v, attn_mask=mask, scale=scale,
                                       enable_gqa=True)
    o = o.transpose(1, 2)
    return torch.where((ctx > 0)[:, None, None, None], o, torch.zeros_like(o))


def varlen_causal_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                          softmax_scale: float | None = None, return_lse: bool = False):
    """Packed causal prefill: q [T, Hq, D], k/v [T, Hkv, D], sequences
    cu_seqlens[s]..cu_seqlens[s+1]; each is the reference's
    F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    (model.py:56-57) in fp32. Returns fp32 [T, Hq, D] (and lse [T, Hq])."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else softmax_scale
    out = torch.zeros(T, Hq, D, dtype=torch.float32)
    lse = torch.full((T, Hq), float("-inf"))
    for s in range(cu_seqlens.numel() - 1):
        a, b = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        if b <= a:
            continue
        qs = q[a:b].float().transpose(0, 1)[None]
        ks = k[a:b].float().transpose(0, 1)[None]
        vs = v[a:b].float().transpose(0, 1)[None]
        o = F.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=scale, enable_gqa=True)
        out[a:b] = o[0].transpose(0, 1)
        if return_lse:
            kr = ks[0].repeat_interleave(Hq // Hkv, dim=0)
            sc = torch.einsum("hid,hjd->hij", qs[0], kr) * scale
            L = b - a
            causal = torch.ones(L, L, dtype=torch.bool).tril()
            sc = sc.masked_fill(~causal, float("-inf"))
            lse[a:b] = torch.logsumexp(sc, dim=-1).transpose(0, 1)
    return (out, lse) if return_lse else out


def paged_chunk_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                        cache_seqlens: torch.Tensor, cu_seqlens_q: torch.Tensor, softmax_scale: float | None = None,
                        causal: bool = True, return_lse: bool = False):
    """Chunked prefill over the paged cache: sequence s has the n_s query
    tokens q[cu_seqlens_q[s]:cu_seqlens_q[s+1]] ([T, Hq, D] packed) and the
    K_s = cache_seqlens[s] keys 0..K_s-1 gathered through its block-table row
    (the chunk's own keys already written there). Causal masking is
    bottom-right aligned, the flash_attn_with_kvcache contract for q_len > 1
    at model.py:60-67: query i sees key j iff j <= i + K_s - n_s. A row that
    sees no key yields zeros (lse -inf). fp32; returns [T, Hq, D] (and lse
    [T, Hq])."""
    T, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else softmax_scale
    out = torch.zeros(T, Hq, D, dtype=torch.float32)
    lse = torch.full((T, Hq), float("-inf"))
    for s in range(cu_seqlens_q.numel() - 1):
        a, b = int(cu_seqlens_q[s]), int(cu_seqlens_q[s + 1])
        n, K = b - a, int(cache_seqlens[s])
        if n <= 0 or K <= 0:
            continue
        k, v = gather_kv(k_cache, v_cache, block_table[s], K)
        kr = k.float().transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)  # [Hq, K, D]
        vr = v.float().transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)
        sc = torch.einsum("ihd,hjd->hij", q[a:b].float(), kr) * scale  # [Hq, n, K]
        if causal:
            vis = torch.arange(K)[None, :] <= (torch.arange(n)[:, None] + (K - n))
            sc = sc.masked_fill(~vis[None], float("-inf"))
        rl = torch.logsumexp(sc, dim=-1)  # [Hq, n]
        pr = torch.exp(sc - torch.where(torch.isfinite(rl), rl, torch.zeros_like(rl))[..., None])
        out[a:b] = torch.einsum("hij,hjd->ihd", pr, vr)
        lse[a:b] = rl.transpose(0, 1)
    return (out, lse) if return_lse else out
