"""lean_infer_b200 — B200-native (sm_100a) paged-attention backend for the
lean-infer Qwen3 engine.

Public API (the drop-ins for the reference's attention path):
  flash_attn_with_kvcache     paged decode attention (kernel b + combine)
  flash_attn_varlen_func      causal varlen prefill attention (kernel c)
  qk_norm_rope_paged_write    fused QK-RMSNorm + RoPE + paged KV write (kernel a)
  paged_kv_write              plain paged KV write (BlockCache.write)
  BlockCache, BlockAllocator  the engine's pool layout and allocator
The kernels live in _lib/liblean_attn.so (C ABI: include/lean_attn.h).
"""
from .flash_attn_interface import (  # noqa: F401
    check_device_errors,
    ensure_init,
    flash_attn_varlen_func,
    flash_attn_with_kvcache,
    paged_kv_write,
    qk_norm_rope_paged_write,
    rope_tables,
    scaled_dot_product_attention,
)
from .cache import BlockAllocator, BlockCache, blocks_for  # noqa: F401

__all__ = [
    "flash_attn_with_kvcache",
    "flash_attn_varlen_func",
    "scaled_dot_product_attention",
    "qk_norm_rope_paged_write",
    "paged_kv_write",
    "rope_tables",
    "check_device_errors",
    "ensure_init",
    "BlockCache",
    "BlockAllocator",
    "blocks_for",
]
