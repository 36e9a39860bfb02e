"""Paged decode attention (kernel b + combine) against the fp32 CPU oracle.

Tolerance: max |out - oracle| <= 2e-2 on bf16 outputs (the bound the
reference's attention path is held to), lse within 1e-2."""
import math

import numpy as np
import pytest
import torch

from oracle import paged_attention as opa

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _workloads():
    from lean_infer_b200 import workloads

    return workloads


def run_case(pkg, dev, B, lo, hi, *, bs=256, hq=16, hkv=8, nb=None, seed=0, lengths=None, lse=False,
             check_rows=None):
    W = _workloads()
    w = W.decode_batch(B, lo, hi, num_blocks=nb, block_size=bs, num_q_heads=hq, num_kv_heads=hkv, seed=seed,
                       lengths=lengths)
    out = pkg.flash_attn_with_kvcache(w.q.to(dev), w.k_cache.to(dev), w.v_cache.to(dev),
                                      cache_seqlens=w.cache_seqlens.to(dev), block_table=w.block_table.to(dev),
                                      causal=True, num_splits=1, return_softmax_lse=lse)
    if lse:
        out, lse_d = out
    torch.cuda.synchronize()
    pkg.check_device_errors(dev.index)
    rows = torch.arange(B) if check_rows is None else check_rows
    ref = opa.paged_decode(w.q[rows], w.k_cache, w.v_cache, w.block_table[rows], w.cache_seqlens[rows],
                           return_lse=lse)
    if lse:
        ref, ref_lse = ref
    got = out.cpu().float()[rows]
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err <= TOL, f"max abs err {err}"
    if lse:
        a, b = lse_d.cpu()[rows, :, 0], ref_lse
        fin = torch.isfinite(b)
        assert torch.equal(torch.isfinite(a), fin)
        assert (a[fin] - b[fin]).abs().max().item() <= 1e-2
    return err


def test_config_single_layer_b8(pkg, cuda_dev):
    """B=8, contexts U[512,1024], pool 512 x 256 x 8 x 128, permuted blocks."""
    run_case(pkg, cuda_dev, 8, 512, 1024, nb=512, seed=1)


def test_b128_engine_batch(pkg, cuda_dev):
    run_case(pkg, cuda_dev, 128, 512, 1024, nb=512, seed=2, lse=True)


@pytest.mark.parametrize("ctx", [[1], [15], [16], [17], [255, 256, 257], [1, 2, 3, 4, 5, 1024, 1023, 31, 33]])
def test_edge_lengths(pkg, cuda_dev, ctx):
    L = torch.tensor(ctx, dtype=torch.int64)
    run_case(pkg, cuda_dev, len(ctx), 0, 0, lengths=L, seed=3, lse=True)


def test_empty_rows_are_zero(pkg, cuda_dev):
    L = torch.tensor([0, 100, 0, 7], dtype=torch.int64)
    W = _workloads()
    w = W.decode_batch(4, 0, 0, lengths=L.clamp(min=1), seed=4)
    seq = torch.tensor([0, 100, 0, 7], dtype=torch.int32)
    out, lse = pkg.flash_attn_with_kvcache(w.q.to(cuda_dev), w.k_cache.to(cuda_dev), w.v_cache.to(cuda_dev),
                                           cache_seqlens=seq.to(cuda_dev), block_table=w.block_table.to(cuda_dev),
                                           return_softmax_lse=True)
    torch.cuda.synchronize()
    out, lse = out.cpu(), lse.cpu()
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0
    assert torch.isneginf(lse[0]).all() and torch.isneginf(lse[2]).all()
    ref = opa.paged_decode(w.q, w.k_cache, w.v_cache, w.block_table, seq)
    assert (out.float() - ref).abs().max().item() <= TOL


@pytest.mark.parametrize("B", [256, 257, 300])
def test_many_short_sequences(pkg, cuda_dev, B):
    """More sequences than CTAs: most are finished inside one CTA. Up to 256
    sequences the split is computed from lengths held in registers, above
    that by the scan over the lengths in memory: both sides of the edge."""
    run_case(pkg, cuda_dev, B, 1, 300, nb=None, seed=5)


@pytest.mark.parametrize("bs", [16, 32, 64, 128])
def test_block_sizes(pkg, cuda_dev, bs):
    run_case(pkg, cuda_dev, 16, 100, 2000, bs=bs, nb=None, seed=6 + bs)


@pytest.mark.parametrize("hkv", [1, 2, 4])
def test_kv_head_shards(pkg, cuda_dev, hkv):
    """Fewer kv heads per call (a KV-head-sharded rank holds 8/P heads)."""
    run_case(pkg, cuda_dev, 24, 1, 1500, hq=2 * hkv, hkv=hkv, nb=None, seed=20 + hkv, lse=True)


@pytest.mark.parametrize("group", [1, 4, 8])
def test_gqa_group_sizes(pkg, cuda_dev, group):
    run_case(pkg, cuda_dev, 12, 1, 900, hq=8 * group, hkv=8, nb=None, seed=30 + group)


def test_long_context_split(pkg, cuda_dev):
    """B=32, contexts U[8192, 32768]: every sequence spans several CTAs."""
    rows = torch.tensor([0, 7, 13, 31])
    run_case(pkg, cuda_dev, 32, 8192, 32768, nb=None, seed=40, check_rows=rows, lse=True)


def test_long_context_block16(pkg, cuda_dev):
    rows = torch.tensor([1, 2, 30])
    run_case(pkg, cuda_dev, 32, 8192, 32768, bs=16, nb=None, seed=41, check_rows=rows)


def test_strided_q_view(pkg, cuda_dev):
    """q as the engine passes it: a transpose(1, 2) view of [B, H, 1, D]."""
    W = _workloads()
    w = W.decode_batch(6, 200, 700, seed=7)
    qt = w.q.transpose(1, 2).contiguous().transpose(1, 2)  # same values, head-major memory
    out = pkg.flash_attn_with_kvcache(qt.to(cuda_dev), w.k_cache.to(cuda_dev), w.v_cache.to(cuda_dev),
                                      cache_seqlens=w.cache_seqlens.to(cuda_dev),
                                      block_table=w.block_table.to(cuda_dev), causal=True)
    ref = opa.paged_decode(w.q, w.k_cache, w.v_cache, w.block_table, w.cache_seqlens)
    assert (out.cpu().float() - ref).abs().max().item() <= TOL


def test_nonfinite_tail_is_masked(pkg, cuda_dev):
    """Pool rows past cache_seqlens holding NaN/Inf must not leak into the output."""
    W = _workloads()
    w = W.decode_batch(4, 0, 0, lengths=torch.tensor([5, 17, 250, 300]), num_blocks=None, seed=8)
    kc, vc = w.k_cache.clone(), w.v_cache.clone()
    for b in range(4):
        L = int(w.cache_seqlens[b])
        for t in range(L, ((L + 255) // 256) * 256):
            blk = int(w.block_table[b, t // 256])
            kc[blk, t % 256] = float("nan")
            vc[blk, t % 256] = float("inf")
    out = pkg.flash_attn_with_kvcache(w.q.to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev),
                                      cache_seqlens=w.cache_seqlens.to(cuda_dev), block_table=w.block_table.to(cuda_dev))
    got = out.cpu().float()
    assert torch.isfinite(got).all()
    ref = opa.paged_decode(w.q, kc, vc, w.block_table, w.cache_seqlens)
    assert (got - ref).abs().max().item() <= TOL


def test_pinned_by_reference_prefill(pkg, cuda_dev):
    """Decode at position t equals row t of the reference's own fp32 causal
    SDPA prefill output (golden fixture), through permuted 16-token blocks."""
    g = dict(np.load(GOLDEN / "attention_prefill.npz"))
    q = torch.from_numpy(g["q"]).transpose(0, 1).to(torch.bfloat16)  # [L, Hq, D]
    k = torch.from_numpy(g["k"]).transpose(0, 1).to(torch.bfloat16)
    v = torch.from_numpy(g["v"]).transpose(0, 1).to(torch.bfloat16)
    o = torch.from_numpy(g["o"]).transpose(0, 1)
    L, bs = q.shape[0], 16
    nblk = -(-L // bs)
    perm = torch.randperm(nblk + 2, generator=torch.Generator().manual_seed(9))[:nblk] + 1
    kc = torch.zeros(nblk + 3, bs, 8, 128, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    for i in range(nblk):
        n = min(bs, L - i * bs)
        kc[perm[i], :n] = k[i * bs: i * bs + n]
        vc[perm[i], :n] = v[i * bs: i * bs + n]
    bt = perm.view(1, -1).expand(L, -1).contiguous().int()
    seq = torch.arange(1, L + 1, dtype=torch.int32)
    out = pkg.flash_attn_with_kvcache(q.view(L, 1, 16, 128).to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev),
                                      cache_seqlens=seq.to(cuda_dev), block_table=bt.to(cuda_dev), causal=True)
    err = (out.cpu().float()[:, 0] - o).abs().max().item()
    assert err <= TOL, err


def test_bad_block_id_reported(pkg, cuda_dev):
    W = _workloads()
    w = W.decode_batch(2, 300, 300, num_blocks=8, seed=10)
    bt = w.block_table.clone()
    bt[1, 1] = 10_000  # outside the pool: read as zeros, reported
    pkg.flash_attn_with_kvcache(w.q.to(cuda_dev), w.k_cache.to(cuda_dev), w.v_cache.to(cuda_dev),
                                cache_seqlens=w.cache_seqlens.to(cuda_dev), block_table=bt.to(cuda_dev))
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="block id"):
        pkg.check_device_errors(cuda_dev.index)


def test_cuda_graph_capture_and_replay(pkg, cuda_dev):
    """The decode call captures into a CUDA graph (no allocation, no host
    sync, device-side split decisions) and replays with new lengths/tables."""
    W = _workloads()
    w1 = W.decode_batch(64, 300, 1000, num_blocks=512, seed=11)
    w2 = W.decode_batch(64, 1, 1024, num_blocks=512, seed=12)
    q = w1.q.to(cuda_dev)
    kc, vc = w1.k_cache.to(cuda_dev), w1.v_cache.to(cuda_dev)
    bt = torch.zeros(64, 4, dtype=torch.int32, device=cuda_dev)
    seq = torch.ones(64, dtype=torch.int32, device=cuda_dev)
    bt[:, : w1.block_table.shape[1]].copy_(w1.block_table)
    seq.copy_(w1.cache_seqlens)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            pkg.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seq, block_table=bt, causal=True)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = pkg.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seq, block_table=bt, causal=True)
    for w in (w1, w2):
        bt.zero_()
        bt[:, : w.block_table.shape[1]].copy_(w.block_table)
        seq.copy_(w.cache_seqlens)
        graph.replay()
        torch.cuda.synchronize()
        ref = opa.paged_decode(w1.q, w1.k_cache, w1.v_cache, w.block_table, w.cache_seqlens)
        assert (out.cpu().float() - ref).abs().max().item() <= TOL
    del graph


def test_matches_flash_attn_with_kvcache(pkg, cuda_dev):
    """Against the reference's own decode kernel, flash_attn_with_kvcache
    (flash-attn 2.8.3), called exactly as model.py:60-67 calls it."""
    fa = pytest.importorskip("flash_attn")
    W = _workloads()
    for B, seed in ((8, 61), (128, 62)):
        w = W.decode_batch(B, 512, 1024, num_blocks=512, seed=seed, device=cuda_dev)
        kw = dict(cache_seqlens=w.cache_seqlens, block_table=w.block_table, causal=True, num_splits=1)
        try:
            ref = fa.flash_attn_with_kvcache(w.q, w.k_cache, w.v_cache, **kw)
        except RuntimeError as e:  # e.g. no kernel image for this GPU in the wheel
            pytest.skip(f"flash_attn_with_kvcache does not run here: {e}")
        out = pkg.flash_attn_with_kvcache(w.q, w.k_cache, w.v_cache, **kw)
        torch.cuda.synchronize()
        assert (out.float() - ref.float()).abs().max().item() <= TOL
