"""Drop-in attention entry points backed by liblean_attn.so (sm_100a).

``flash_attn_with_kvcache`` keeps the keyword signature of
flash_attn.flash_attn_with_kvcache (flash-attn 2.8.3, the function the engine
imports at leaninfer/qwen3/model.py:3 and calls at model.py:60-67) for the
arguments that call site and the engine's CUDA-graph decode use: paged
k_cache/v_cache, block_table, cache_seqlens, softmax_scale, causal,
num_splits, return_softmax_lse. Arguments the engine never passes (in-place
append of new k/v, rotary, cache_batch_idx, leftpad, sliding window, softcap,
alibi) raise NotImplementedError instead of being silently ignored.

Host rules shared by every entry point here:
  * tensors must be CUDA bf16 (indices int32, positions int64) on one device;
  * the kernels launch on torch's current stream for that device;
  * nothing here synchronises the host, and the only allocations are the
    output tensors and a per-device workspace that is created on the first
    call and reused (so warm up once before CUDA-graph capture, exactly as
    the engine does for flash-attn at leaninfer/engine/llm_engine.py:51-53).
"""
from __future__ import annotations

import ctypes
import math
import threading
from typing import Optional

import torch

from . import _lib

_state_lock = threading.Lock()
_inited: set[int] = set()
_workspaces: dict[int, torch.Tensor] = {}
_error_words: dict[int, torch.Tensor] = {}
_rope_tables: dict[tuple, tuple[torch.Tensor, torch.Tensor]] = {}


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _device_index(t: torch.Tensor) -> int:
    if t.device.type != "cuda":
        raise RuntimeError("lean_attn kernels need CUDA tensors (there is no CPU path)")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def ensure_init(device: int) -> None:
    """la_init() once per device: kernel attributes and module load, done
    before any graph capture."""
    if device in _inited:
        return
    with _state_lock:
        if device not in _inited:
            _lib.call("la_init", device)
            _inited.add(device)


def error_word(device: int) -> torch.Tensor:
    """The per-device int32 error word the kernels write on device-side faults."""
    w = _error_words.get(device)
    if w is None:
        with _state_lock:
            w = _error_words.get(device)
            if w is None:
                w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", device))
                _error_words[device] = w
    return w


def check_device_errors(device: Optional[int] = None, clear: bool = True) -> None:
    """Synchronise with `device` and raise if a kernel recorded an error."""
    dev = torch.cuda.current_device() if device is None else device
    w = _error_words.get(dev)
    if w is None:
        return
    code = int(w.item())
    if clear:
        w.zero_()
    if code:
        raise _lib.LeanAttnError(f"device error {code}: {_lib.DEVERR_NAMES.get(code, 'unknown')}")


def _workspace(device: int, nbytes: int) -> torch.Tensor:
    """The per-device decode workspace, grown to `nbytes` if needed.

    Its size depends only on head counts and the SM count, so it is created
    by the first call and normally never grows. If it must grow, kernels
    queued earlier (any stream) may still use the old buffer, so the device
    is synchronised before the old tensor is dropped; growing inside a CUDA
    graph capture is refused, since a captured graph would keep the freed
    pointer (warm up with the largest head count before capturing)."""
    ws = _workspaces.get(device)
    if ws is None or ws.numel() < nbytes:
        with _state_lock:
            ws = _workspaces.get(device)
            if ws is None or ws.numel() < nbytes:
                if ws is not None:
                    if torch.cuda.is_current_stream_capturing():
                        raise RuntimeError("the decode workspace must grow during a CUDA graph capture: call "
                                           "once with these head counts before capturing")
                    torch.cuda.synchronize(device)
                ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", device))
                _workspaces[device] = ws
    return ws


def decode_workspace_bytes(device: int, num_q_heads: int, num_kv_heads: int, head_dim: int) -> int:
    n = ctypes.c_size_t(0)
    _lib.call("la_paged_decode_workspace_size", device, num_q_heads, num_kv_heads, head_dim, ctypes.byref(n))
    return int(n.value)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


# --------------------------------------------------------------------------
# (b) decode
# --------------------------------------------------------------------------
def flash_attn_with_kvcache(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k: Optional[torch.Tensor] = None,
    v: Optional[torch.Tensor] = None,
    rotary_cos: Optional[torch.Tensor] = None,
    rotary_sin: Optional[torch.Tensor] = None,
    cache_seqlens=None,
    cache_batch_idx: Optional[torch.Tensor] = None,
    cache_leftpad: Optional[torch.Tensor] = None,
    block_table: Optional[torch.Tensor] = None,
    softmax_scale: Optional[float] = None,
    causal: bool = False,
    window_size=(-1, -1),
    softcap: float = 0.0,
    rotary_interleaved: bool = True,
    alibi_slopes: Optional[torch.Tensor] = None,
    num_splits: int = 0,
    return_softmax_lse: bool = False,
):
    """Paged GQA attention over the KV cache.

    One query token per sequence (decode, q [B, 1, Hq, D]) runs the split-KV
    decode kernel. q_len > 1 (chunked prefill, q [B, Sq, Hq, D], the chunk's
    keys already in the cache) runs the tcgen05 prefill kernel over the paged
    keys, causal masking bottom-right aligned (query i sees keys
    0..cache_seqlens[b] - Sq + i); block_size then a multiple of 128, or
    16, 32 or 64.

    q: [B, Sq, Hq, D] bf16. k_cache / v_cache: [num_blocks, block_size, Hkv, D]
    bf16 with block_table [B, max_blocks] int32, or [B, S, Hkv, D] without a
    block table. cache_seqlens: [B] int32 (or an int for all rows).
    Returns out [B, Sq, Hq, D] (and softmax_lse [B, Hq, Sq] fp32 when asked).

    causal is accepted and has no effect at one query token (bottom-right
    alignment lets the query see all cache_seqlens[b] keys). num_splits is a
    hint only: the split of every sequence across SMs is chosen on the device
    from cache_seqlens so the launch stays capturable; results do not depend
    on it beyond fp32 summation order.
    """
    if k is not None or v is not None:
        raise NotImplementedError("in-place append of new k/v: write the cache with qk_norm_rope_paged_write")
    if rotary_cos is not None or rotary_sin is not None:
        raise NotImplementedError("rotary inside attention: rope is fused into qk_norm_rope_paged_write")
    if cache_batch_idx is not None or cache_leftpad is not None:
        raise NotImplementedError("cache_batch_idx / cache_leftpad")
    if tuple(window_size) != (-1, -1) or softcap != 0.0 or alibi_slopes is not None:
        raise NotImplementedError("sliding window / softcap / alibi")
    _check(q.dim() == 4, "q must be [batch, seqlen_q, num_heads, head_dim]")
    B, Sq, Hq, D = q.shape
    _check(q.dtype == torch.bfloat16 and k_cache.dtype == torch.bfloat16 and v_cache.dtype == torch.bfloat16,
           "q, k_cache and v_cache must be bfloat16")
    _check(k_cache.shape == v_cache.shape and k_cache.stride() == v_cache.stride(),
           "k_cache and v_cache must have the same shape and strides")
    _check(k_cache.dim() == 4, "k_cache must be 4-D")
    dev = _device_index(q)
    _check(k_cache.device == q.device and v_cache.device == q.device, "all tensors must be on one device")
    _check(q.stride(-1) == 1 and k_cache.stride(-1) == 1, "the head_dim axis must be contiguous")
    Hkv = k_cache.shape[2]
    _check(k_cache.shape[3] == D, "head_dim of q and k_cache differ")
    _check(Hq % Hkv == 0, "num_heads must be a multiple of num_heads_k")

    if block_table is None:
        _check(k_cache.shape[0] == B, "without block_table k_cache must be [batch, seqlen, Hkv, D]")
        block_table = _identity_table(B, q.device)
    _check(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.shape[0] == B,
           "block_table must be int32 [batch, max_blocks]")
    _check(block_table.device == q.device and block_table.stride(1) == 1, "block_table must be row-contiguous on q's device")
    if cache_seqlens is None:
        cache_seqlens = torch.full((B,), k_cache.shape[1] * block_table.shape[1], dtype=torch.int32, device=q.device)
    elif isinstance(cache_seqlens, int):
        cache_seqlens = torch.full((B,), cache_seqlens, dtype=torch.int32, device=q.device)
    _check(cache_seqlens.dtype == torch.int32 and cache_seqlens.numel() == B and cache_seqlens.is_contiguous(),
           "cache_seqlens must be a contiguous int32 [batch] tensor")
    _check(cache_seqlens.device == q.device, "cache_seqlens must be on q's device")

    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    if Sq != 1:
        if q.stride(0) != Sq * q.stride(1):
            q = q.contiguous()
        out = torch.empty((B, Sq, Hq, D), dtype=q.dtype, device=q.device)
        lse = torch.empty((Hq, B * Sq), dtype=torch.float32, device=q.device) if return_softmax_lse else None
        if B > 0 and Sq > 0:
            _prefill_paged(dev, q.stride(1), q.stride(2), q, k_cache, v_cache, block_table, cache_seqlens, None, Sq, B,
                           Sq, B * Sq, Hq, Hkv, D, scale, causal, out, out.stride(1), out.stride(2), lse)
        if return_softmax_lse:
            return out, lse.view(Hq, B, Sq).permute(1, 0, 2)
        return out
    out = torch.empty((B, 1, Hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, Hq, 1), dtype=torch.float32, device=q.device) if return_softmax_lse else None
    if B == 0:
        return (out, lse) if return_softmax_lse else out

    with torch.cuda.device(dev):
        ensure_init(dev)
        need = decode_workspace_bytes(dev, Hq, Hkv, D)
        ws = _workspace(dev, need)
        err = error_word(dev)
        _lib.call(
            "la_paged_decode",
            _ptr(q), q.stride(0), q.stride(2),
            _ptr(k_cache), _ptr(v_cache),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            k_cache.shape[0], k_cache.shape[1],
            _ptr(block_table), block_table.stride(0), block_table.shape[1],
            _ptr(cache_seqlens),
            B, Hq, Hkv, D,
            ctypes.c_float(scale),
            _ptr(out), out.stride(0), out.stride(2),
            _ptr(lse),
            _ptr(ws), ws.numel(),
            _ptr(err), _stream(q.device),
        )
    return (out, lse) if return_softmax_lse else out


def _prefill_paged(dev, q_ts, q_hs, q, k_cache, v_cache, block_table, k_lens, cu_q, q_len, S, max_q, T, Hq, Hkv, D,
                   scale, causal, out, o_ts, o_hs, lse):
    """la_prefill_paged on q's stream (chunked prefill over the paged cache)."""
    with torch.cuda.device(dev):
        ensure_init(dev)
        _lib.call(
            "la_prefill_paged",
            _ptr(q), q_ts, q_hs,
            _ptr(k_cache), _ptr(v_cache),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            k_cache.shape[0], k_cache.shape[1],
            _ptr(block_table), block_table.stride(0), block_table.shape[1],
            _ptr(k_lens),
            _ptr(cu_q), q_len, S, max_q, T,
            Hq, Hkv, D,
            ctypes.c_float(scale), 1 if causal else 0,
            _ptr(out), o_ts, o_hs,
            _ptr(lse),
            _ptr(error_word(dev)), _stream(q.device),
        )


_identity_tables: dict[tuple, torch.Tensor] = {}


def _identity_table(B: int, device: torch.device) -> torch.Tensor:
    key = (B, device)
    t = _identity_tables.get(key)
    if t is None:
        t = torch.arange(B, dtype=torch.int32, device=device).view(B, 1)
        _identity_tables[key] = t
    return t


# --------------------------------------------------------------------------
# (a) fused QK-RMSNorm + RoPE + paged KV write
# --------------------------------------------------------------------------
def rope_tables(max_pos: int, head_dim: int, theta: float, device, dtype=torch.bfloat16):
    """cos/sin tables [max_pos, head_dim/2] by the reference formula.

    leaninfer/qwen3/layers.py:7-15 builds, per forward, inv_freq in fp32,
    angles = float(pos + t) * inv_freq, cat(angles, angles).cos().to(dtype).
    The table holds the same values indexed by absolute position (only the
    first half: the second is a copy). Built once per (device, theta, D) and
    grown on demand, on the device, with torch's own cos/sin so the values are
    the ones the reference computes on that device.
    """
    device = torch.device(device)
    key = (device, float(theta), int(head_dim), dtype)
    cur = _rope_tables.get(key)
    if cur is not None and cur[0].shape[0] >= max_pos:
        return cur[0][:max_pos], cur[1][:max_pos]
    n = max(max_pos, 4096 if cur is None else 2 * cur[0].shape[0])
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    angles = torch.arange(n, device=device).float()[:, None] * inv_freq[None, :]
    tabs = (angles.cos().to(dtype).contiguous(), angles.sin().to(dtype).contiguous())
    _rope_tables[key] = tabs
    return tabs[0][:max_pos], tabs[1][:max_pos]


def _tokens_view(x: torch.Tensor, name: str) -> torch.Tensor:
    """[T, H, D] view of a [T, H, D] or [B, n, H, D] tensor (no copy)."""
    if x.dim() == 3:
        return x
    _check(x.dim() == 4, f"{name} must be [tokens, heads, D] or [batch, q_len, heads, D]")
    B, n, H, D = x.shape
    if n == 1 or x.stride(0) == n * x.stride(1):
        return x.as_strided((B * n, H, D), (x.stride(1) if n > 1 else x.stride(0), x.stride(2), x.stride(3)))
    raise RuntimeError(f"{name}: batch and q_len axes cannot be merged without a copy")


def qk_norm_rope_paged_write(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_norm_weight: torch.Tensor,
    k_norm_weight: torch.Tensor,
    rope_cos: torch.Tensor,
    rope_sin: torch.Tensor,
    pos: torch.Tensor,
    block_table: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    eps: float = 1e-6,
    cu_seqlens: Optional[torch.Tensor] = None,
    q_out: Optional[torch.Tensor] = None,
    k_out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Fused q_norm/k_norm + RoPE + cache.write for one layer; returns q_out
    (and writes the rotated k to k_out as well when given).

    q: [T, Hq, D] (or [B, n, Hq, D]); k, v: [T, Hkv, D] (or [B, n, Hkv, D]),
    the raw projections. pos: int64 [num_seqs] start position of each
    sequence (the reference's `pos`). Without cu_seqlens the tokens are
    num_seqs rows of q_len = T / num_seqs; with cu_seqlens (int32
    [num_seqs+1]) they are packed varlen sequences. k_cache / v_cache:
    [num_blocks, block_size, Hkv, D] (a layer slice of the pool).
    """
    nseq = pos.shape[0]
    q_len = 0
    if q.dim() == 4:
        q_len = q.shape[1]
    q3, k3, v3 = _tokens_view(q, "q"), _tokens_view(k, "k"), _tokens_view(v, "v")
    T, Hq, D = q3.shape
    Hkv = k3.shape[1]
    _check(k3.shape[0] == T and v3.shape[0] == T and v3.shape[1] == Hkv, "q, k, v token counts differ")
    for name, t in (("q", q3), ("k", k3), ("v", v3), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("q_norm_weight", q_norm_weight), ("k_norm_weight", k_norm_weight),
                    ("rope_cos", rope_cos), ("rope_sin", rope_sin)):
        _check(t.dtype == torch.bfloat16, f"{name} must be bfloat16")
        _check(t.stride(-1) == 1, f"{name}: last axis must be contiguous")
    _check(pos.dtype == torch.int64, "pos must be int64")
    _check(block_table.dtype == torch.int32 and block_table.stride(-1) == 1, "block_table must be int32")
    _check(k_cache.shape == v_cache.shape and k_cache.stride() == v_cache.stride(), "k_cache/v_cache mismatch")
    _check(rope_cos.is_contiguous() and rope_sin.is_contiguous() and rope_cos.shape == rope_sin.shape
           and rope_cos.shape[1] == D // 2, "rope tables must be contiguous [max_pos, D/2]")
    if cu_seqlens is None:
        if q_len == 0:
            _check(nseq > 0 and T % nseq == 0, "tokens must split evenly over sequences")
            q_len = T // nseq if nseq else 1
    else:
        _check(cu_seqlens.dtype == torch.int32 and cu_seqlens.numel() == nseq + 1, "cu_seqlens must be int32 [num_seqs+1]")
    if q_out is None:
        q_out = torch.empty((T, Hq, D), dtype=q.dtype, device=q.device)
    qo = _tokens_view(q_out, "q_out")
    ko = None
    if k_out is not None:
        ko = _tokens_view(k_out, "k_out")
        _check(ko.shape == k3.shape and ko.dtype == torch.bfloat16 and ko.stride(-1) == 1, "k_out must match k")
    dev = _device_index(q)
    with torch.cuda.device(dev):
        ensure_init(dev)
        _lib.call(
            "la_qk_norm_rope_paged_write",
            _ptr(q3), q3.stride(0), q3.stride(1),
            _ptr(k3), k3.stride(0), k3.stride(1),
            _ptr(v3), v3.stride(0), v3.stride(1),
            _ptr(q_norm_weight), _ptr(k_norm_weight), ctypes.c_float(eps),
            _ptr(rope_cos), _ptr(rope_sin), rope_cos.shape[0],
            _ptr(pos), _ptr(cu_seqlens),
            nseq, q_len, T,
            _ptr(block_table), block_table.stride(0), block_table.shape[1],
            _ptr(k_cache), _ptr(v_cache),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            k_cache.shape[0], k_cache.shape[1],
            _ptr(qo), qo.stride(0), qo.stride(1),
            _ptr(ko), ko.stride(0) if ko is not None else 0, ko.stride(1) if ko is not None else 0,
            Hq, Hkv, D,
            _ptr(error_word(dev)), _stream(q.device),
        )
    return q_out


def paged_kv_write(
    k: torch.Tensor,
    v: torch.Tensor,
    pos: torch.Tensor,
    block_table: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cu_seqlens: Optional[torch.Tensor] = None,
) -> None:
    """Scatter k, v ([T, Hkv, D] or [B, n, Hkv, D]) into the paged cache: the
    device form of BlockCache.write (leaninfer/engine/cache_manager.py:63-76)."""
    nseq = pos.shape[0]
    q_len = k.shape[1] if k.dim() == 4 else 0
    k3, v3 = _tokens_view(k, "k"), _tokens_view(v, "v")
    T, Hkv, D = k3.shape
    for name, t in (("k", k3), ("v", v3), ("k_cache", k_cache), ("v_cache", v_cache)):
        _check(t.dtype == torch.bfloat16 and t.stride(-1) == 1, f"{name} must be bf16 with a contiguous last axis")
    _check(pos.dtype == torch.int64 and block_table.dtype == torch.int32, "pos int64, block_table int32")
    _check(k_cache.shape == v_cache.shape and k_cache.stride() == v_cache.stride(), "k_cache/v_cache mismatch")
    if cu_seqlens is None and q_len == 0:
        _check(nseq > 0 and T % nseq == 0, "tokens must split evenly over sequences")
        q_len = T // nseq
    dev = _device_index(k)
    with torch.cuda.device(dev):
        ensure_init(dev)
        _lib.call(
            "la_paged_kv_write",
            _ptr(k3), k3.stride(0), k3.stride(1),
            _ptr(v3), v3.stride(0), v3.stride(1),
            _ptr(pos), _ptr(cu_seqlens),
            nseq, q_len, T,
            _ptr(block_table), block_table.stride(0), block_table.shape[1],
            _ptr(k_cache), _ptr(v_cache),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            k_cache.shape[0], k_cache.shape[1],
            Hkv, D,
            _ptr(error_word(dev)), _stream(k.device),
        )


# --------------------------------------------------------------------------
# (c) causal varlen prefill
# --------------------------------------------------------------------------
def flash_attn_varlen_func(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    max_seqlen_q: int,
    max_seqlen_k: int,
    dropout_p: float = 0.0,
    softmax_scale: Optional[float] = None,
    causal: bool = False,
    window_size=(-1, -1),
    softcap: float = 0.0,
    alibi_slopes: Optional[torch.Tensor] = None,
    deterministic: bool = False,
    return_attn_probs: bool = False,
    block_table: Optional[torch.Tensor] = None,
    return_softmax_lse: bool = False,
):
    """Packed attention over varlen sequences (flash-attn 2.8.3 varlen
    signature): q [T, Hq, D] bf16, cu_seqlens_q int32 [S+1].

    Without block_table, k/v [T, Hkv, D] are the same tokens as the queries
    (prefill self-attention): cu_seqlens_k must be cu_seqlens_q. With
    block_table [S, max_blocks] int32, k/v are the paged caches
    [num_blocks, block_size, Hkv, D] and sequence s has
    cu_seqlens_k[s+1] - cu_seqlens_k[s] keys there (chunked prefill: causal
    masking bottom-right aligned). Returns out [T, Hq, D] (and lse [Hq, T]
    fp32 when return_softmax_lse)."""
    if dropout_p != 0.0 or tuple(window_size) != (-1, -1) or softcap != 0.0 or alibi_slopes is not None:
        raise NotImplementedError("dropout / sliding window / softcap / alibi")
    if return_attn_probs:
        raise NotImplementedError("return_attn_probs")
    if block_table is not None:
        return _varlen_paged(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale, causal, block_table,
                             return_softmax_lse)
    if cu_seqlens_k is not cu_seqlens_q and cu_seqlens_k.data_ptr() != cu_seqlens_q.data_ptr():
        # distinct tensors: compare the values (a device sync; pass one tensor
        # twice, as prefill does, to avoid it)
        if cu_seqlens_k.shape != cu_seqlens_q.shape or not torch.equal(cu_seqlens_k, cu_seqlens_q):
            raise NotImplementedError("cross-attention (cu_seqlens_k != cu_seqlens_q)")
    _check(q.dim() == 3 and k.dim() == 3 and v.dim() == 3, "q/k/v must be [total_tokens, heads, head_dim]")
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    _check(k.shape[0] == T and v.shape == k.shape and k.shape[2] == D, "q/k/v shapes differ")
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check(t.dtype == torch.bfloat16 and t.stride(-1) == 1, f"{name} must be bf16 with a contiguous last axis")
    _check(cu_seqlens_q.dtype == torch.int32 and cu_seqlens_q.is_contiguous(), "cu_seqlens must be contiguous int32")
    dev = _device_index(q)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    out = torch.empty((T, Hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((Hq, T), dtype=torch.float32, device=q.device) if return_softmax_lse else None
    S = cu_seqlens_q.numel() - 1
    with torch.cuda.device(dev):
        ensure_init(dev)
        _lib.call(
            "la_prefill_varlen",
            _ptr(q), q.stride(0), q.stride(1),
            _ptr(k), k.stride(0), k.stride(1),
            _ptr(v), v.stride(0), v.stride(1),
            _ptr(cu_seqlens_q), S, int(max(max_seqlen_q, max_seqlen_k)), T,
            Hq, Hkv, D,
            ctypes.c_float(scale), 1 if causal else 0,
            _ptr(out), out.stride(0), out.stride(1),
            _ptr(lse),
            _ptr(error_word(dev)), _stream(q.device),
        )
    return (out, lse) if return_softmax_lse else out


def _varlen_paged(q, k_cache, v_cache, cu_q, cu_k, max_seqlen_q, softmax_scale, causal, block_table, return_lse):
    _check(q.dim() == 3 and k_cache.dim() == 4 and v_cache.shape == k_cache.shape
           and k_cache.stride() == v_cache.stride(), "paged varlen: q [T, Hq, D], k/v caches [NB, BS, Hkv, D]")
    T, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache)):
        _check(t.dtype == torch.bfloat16 and t.stride(-1) == 1, f"{name} must be bf16 with a contiguous last axis")
    _check(k_cache.shape[3] == D and Hq % Hkv == 0, "head_dim / head counts of q and the caches do not fit")
    _check(cu_q.dtype == torch.int32 and cu_q.is_contiguous() and cu_k.dtype == torch.int32
           and cu_k.shape == cu_q.shape, "cu_seqlens must be int32 [S+1]")
    S = cu_q.numel() - 1
    _check(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.shape[0] == S
           and block_table.stride(1) == 1, "block_table must be int32 [S, max_blocks], row-contiguous")
    dev = _device_index(q)
    k_lens = (cu_k[1:] - cu_k[:-1]).to(torch.int32)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    out = torch.empty((T, Hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((Hq, T), dtype=torch.float32, device=q.device) if return_lse else None
    if S > 0 and T > 0:
        _prefill_paged(dev, q.stride(0), q.stride(1), q, k_cache, v_cache, block_table, k_lens, cu_q, 0, S,
                       int(max_seqlen_q), T, Hq, Hkv, D, scale, causal, out, out.stride(0), out.stride(1), lse)
    return (out, lse) if return_lse else out


_uniform_cu: dict[tuple, torch.Tensor] = {}


def _uniform_cu_for(B: int, L: int, device) -> torch.Tensor:
    """cu_seqlens [0, L, 2L, ..., BL] int32 on `device`, cached per shape."""
    key = (B, L, device)
    cu = _uniform_cu.get(key)
    if cu is None:
        cu = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device=device)
        _uniform_cu[key] = cu
    return cu


def scaled_dot_product_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_mask=None,
                                 dropout_p: float = 0.0, is_causal: bool = False, scale: Optional[float] = None,
                                 enable_gqa: bool = False) -> torch.Tensor:
    """Drop-in for the prefill call F.scaled_dot_product_attention(q, k, v,
    is_causal=True, enable_gqa=True) at leaninfer/qwen3/model.py:57:
    q [B, Hq, L, D], k/v [B, Hkv, L, D] bf16 -> [B, Hq, L, D]. Runs the varlen
    kernel with B sequences of length L (no copy when the [B, L, H, D] memory
    order of the engine's transposed projections is contiguous)."""
    if attn_mask is not None or dropout_p != 0.0:
        raise NotImplementedError("attn_mask / dropout")
    B, Hq, L, D = q.shape
    Hkv = k.shape[1]
    if Hq != Hkv and not enable_gqa:
        raise RuntimeError("Hq != Hkv requires enable_gqa=True")
    qt, kt, vt = (x.transpose(1, 2) for x in (q, k, v))  # [B, L, H, D]
    if B == 1:
        # One sequence (the reference's prefill): the kernel takes the token
        # and head strides as they are, so the [1, H, L, D] tensors need no copy.
        cu = _uniform_cu_for(1, L, q.device)
        out = flash_attn_varlen_func(qt[0], kt[0], vt[0], cu, cu, L, L, softmax_scale=scale, causal=is_causal)
        return out.view(1, L, Hq, D).transpose(1, 2)
    qt, kt, vt = (x if x.is_contiguous() else x.contiguous() for x in (qt, kt, vt))
    cu = _uniform_cu_for(B, L, q.device)
    out = flash_attn_varlen_func(qt.view(B * L, Hq, D), kt.view(B * L, Hkv, D), vt.view(B * L, Hkv, D), cu, cu, L, L,
                                 softmax_scale=scale, causal=is_causal)
    return out.view(B, L, Hq, D).transpose(1, 2)
