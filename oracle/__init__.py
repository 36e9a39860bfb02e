"""CPU oracle for the paged-attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU in fp32 / bf16 torch and numpy, the
reference's algorithm for every op the sm_100a kernels replace:

  pre_attention.py    QK RMSNorm (model.py:43-44, 50-51), build_rope /
                      rotate_half / apply_rope (layers.py:7-23), BlockCache.write
                      and BlockAllocator (cache_manager.py:13-42, 63-76)
  paged_attention.py  decode attention over the paged cache (the
                      flash_attn_with_kvcache call, model.py:58-67, computed as
                      gather-by-block_table + fp32 SDPA) and causal varlen
                      prefill (model.py:56-57)
  qwen3_step.py       the reference model's full decode step in fp32 on the CPU
                      (model.py:25-112), the CPU baseline of the benchmark

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import it, and only as the checker or the timed CPU baseline. The product
path (package lean-infer_b200) never imports or calls anything here; it has no
CPU fallback.

Pinning: tests/golden/make_golden.py runs the reference's own code
(leaninfer.qwen3.model / layers, leaninfer.engine.cache_manager) on the CPU
and stores its inputs and outputs as fixtures; tests/test_oracle.py checks this
oracle against them. The reference has no golden vectors of its own (it has no
tests); the attention itself is flash-attn 2.8.3's, a compiled third-party
dependency, whose contract is restated from its documented semantics and
pinned through the reference's SDPA prefill path (a decode query at position t
must equal row t of the causal prefill output over the same keys).
"""
