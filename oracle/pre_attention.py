"""Oracle for kernel (a): QK RMSNorm + RoPE + paged KV write (CPU).

Test infrastructure only (see oracle/__init__.py).
"""
from __future__ import annotations

from collections import deque

import numpy as np
import torch
import torch.nn.functional as F


# ----------------------------------------------------------------- RMSNorm
def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """nn.RMSNorm(head_dim, eps) as the reference applies it (model.py:43-44,
    50-51): torch's own rms_norm, fp32 internally, one rounding to x.dtype."""
    return F.rms_norm(x, (x.shape[-1],), weight, eps)


def rms_norm_kernel_order(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """The same RMSNorm with the sum of squares taken in the kernel's fixed
    fp32 order: 32 lanes hold 4 consecutive elements each and add their
    squares left to right, then an xor butterfly over offsets 16, 8, 4, 2, 1.
    mean = sum/128, r = 1/sqrt(mean+eps) (correctly rounded), y = (x*r)*w in
    fp32, then one round-to-nearest-even to bf16. Rows of 128 only."""
    assert x.shape[-1] == 128
    shape = x.shape
    xf = x.float().reshape(-1, 128).numpy().astype(np.float32)
    wf = weight.float().numpy().astype(np.float32)
    sq = (xf * xf).astype(np.float32).reshape(-1, 32, 4)
    s = ((sq[..., 0] + sq[..., 1]).astype(np.float32) + sq[..., 2]).astype(np.float32)
    s = (s + sq[..., 3]).astype(np.float32)
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        s = (s + s[:, lanes ^ off]).astype(np.float32)
    s = s[:, 0]
    mean = (s * np.float32(1.0 / 128.0)).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt((mean + np.float32(eps)).astype(np.float32))).astype(np.float32)
    y = ((xf * r[:, None]).astype(np.float32) * wf[None, :]).astype(np.float32)
    return torch.from_numpy(y).to(torch.bfloat16).reshape(shape)


# ----------------------------------------------------------------- RoPE
def inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """layers.py:9: 1 / theta^(arange(0, D, 2)/D) in fp32."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))


def build_rope(pos: torch.Tensor, q_len: int, head_dim: int, theta: float, dtype=torch.bfloat16):
    """layers.py:7-15: cos, sin [B, 1, q_len, D] for rows starting at pos."""
    positions = pos[:, None] + torch.arange(q_len)
    angles = positions[..., None].float() * inv_freq(head_dim, theta)
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos()[:, None].to(dtype), emb.sin()[:, None].to(dtype)


def rope_tables(max_pos: int, head_dim: int, theta: float, dtype=torch.bfloat16):
    """[max_pos, D/2] cos/sin tables holding build_rope's values by absolute
    position (the first half of cat(angles, angles))."""
    angles = torch.arange(max_pos).float()[:, None] * inv_freq(head_dim, theta)[None, :]
    return angles.cos().to(dtype), angles.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """layers.py:18-20."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """layers.py:22-23, in x's dtype (bf16: three roundings)."""
    return x * cos + rotate_half(x) * sin


def rope_from_tables(x: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor, positions: torch.Tensor):
    """apply_rope for x [T, H, D] at absolute positions [T] using the tables."""
    c = cos_tab[positions]  # [T, D/2]
    s = sin_tab[positions]
    c = torch.cat((c, c), dim=-1)[:, None, :]
    s = torch.cat((s, s), dim=-1)[:, None, :]
    return apply_rope(x, c, s)


# ----------------------------------------------------------------- cache
def blocks_for(n_tokens: int, block_size: int) -> int:
    return -(-n_tokens // block_size)


class BlockAllocator:
    """cache_manager.py:13-42: FIFO free list 1..NB-1 (block 0 = trash)."""

    def __init__(self, num_blocks: int) -> None:
        self.free: deque[int] = deque(range(1, num_blocks))

    def allocate(self, n: int) -> list[int]:
        assert n <= len(self.free), f"Insufficient free slots: asked {n}, free {len(self.free)}"
        return [self.free.popleft() for _ in range(n)]

    def release(self, blocks: list[int]) -> None:
        self.free.extend(blocks)


def block_cache_write(k_layer: torch.Tensor, v_layer: torch.Tensor, block_tables: torch.Tensor,
                      pos: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """cache_manager.py:63-76 on one layer slice [NB, BS, Hkv, D].
    k, v: [B, Hkv, q_len, D]."""
    bs = k_layer.shape[1]
    q_len = k.shape[2]
    cols = pos[:, None] + torch.arange(q_len)
    phys = block_tables.long().gather(1, cols // bs)
    off = cols % bs
    k_layer[phys, off] = k.transpose(1, 2)
    v_layer[phys, off] = v.transpose(1, 2)


def token_positions(pos: torch.Tensor, q_len: int | None, cu_seqlens: torch.Tensor | None):
    """(sequence index, absolute position) of every token, in token order."""
    if cu_seqlens is None:
        B = pos.shape[0]
        seq = torch.arange(B).repeat_interleave(q_len)
        t = torch.arange(q_len).repeat(B)
    else:
        lens = (cu_seqlens[1:] - cu_seqlens[:-1]).long()
        seq = torch.arange(len(lens)).repeat_interleave(lens)
        t = torch.arange(int(cu_seqlens[-1])) - cu_seqlens[:-1].long()[seq]
    return seq, pos[seq] + t


def qk_norm_rope_paged_write(q, k, v, q_norm_weight, k_norm_weight, eps, cos_tab, sin_tab, pos, block_table,
                             k_cache, v_cache, q_len=None, cu_seqlens=None, norm="kernel"):
    """Reference of la_qk_norm_rope_paged_write on tokens [T, H, D] (bf16).
    Writes k_cache / v_cache ([NB, BS, Hkv, D]) in place and returns q_out.
    norm="kernel" fixes the kernel's reduction order (bit-exact target);
    norm="reference" uses torch's rms_norm (the reference module)."""
    nf = rms_norm_kernel_order if norm == "kernel" else rms_norm_reference
    seq, positions = token_positions(pos, q_len, cu_seqlens)
    # A negative start position marks an idle sequence: no cache write, zero
    # outputs (the kernel's contract; the reference engine uses a trash block
    # instead, llm_engine.py:67-69).
    idle = torch.as_tensor(pos).long().reshape(-1)[seq] < 0
    positions = torch.where(idle, torch.zeros_like(positions), positions)
    qn = nf(q, q_norm_weight, eps)
    kn = nf(k, k_norm_weight, eps)
    q_out = rope_from_tables(qn, cos_tab, sin_tab, positions)
    k_out = rope_from_tables(kn, cos_tab, sin_tab, positions)
    q_out = torch.where(idle[:, None, None], torch.zeros_like(q_out), q_out)
    k_out = torch.where(idle[:, None, None], torch.zeros_like(k_out), k_out)
    live = ~idle
    bs = k_cache.shape[1]
    phys = block_table.long()[seq[live], positions[live] // bs]
    off = positions[live] % bs
    k_cache[phys, off] = k_out[live]
    v_cache[phys, off] = v[live]
    return q_out, k_out
