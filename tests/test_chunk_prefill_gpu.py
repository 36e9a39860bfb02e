"""Chunked prefill over the paged cache (kernel c with paged keys, through
la_prefill_paged) against the fp32 CPU oracle.

The chunk's queries attend to the keys already in the cache (prefix + the
chunk itself) with bottom-right causal alignment — flash_attn_with_kvcache
with q_len > 1 at model.py:60-67. Tolerance: max |out - oracle| <= 2e-2 on
bf16 outputs; lse within 1e-2."""
import pytest
import torch

from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _pool(nb, bs, hkv, seed, fill_nan=False):
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(nb, bs, hkv, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, bs, hkv, 128, generator=g).to(torch.bfloat16)
    return kc, vc


def _tables(k_lens, bs, seed, spare=3):
    """Block tables for the given key counts from a seeded permutation of
    1..NB-1 (block 0 reserved), with `spare` unused blocks in the pool."""
    need = [max(1, -(-int(n) // bs)) for n in k_lens]
    nb = sum(need) + 1 + spare
    g = torch.Generator().manual_seed(seed + 11)
    perm = (torch.randperm(nb - 1, generator=g) + 1).to(torch.int32)
    bt = torch.zeros(len(need), max(need), dtype=torch.int32)
    o = 0
    for s, n in enumerate(need):
        bt[s, :n] = perm[o:o + n]
        o += n
    return bt, nb


def _nan_tails(kc, vc, bt, k_lens, bs):
    """Fill every pool slot that holds no key of any sequence with NaN."""
    used = torch.zeros(kc.shape[0], bs, dtype=torch.bool)
    for s, K in enumerate(k_lens):
        for t in range(int(K)):
            used[int(bt[s, t // bs]), t % bs] = True
    kc = kc.clone()
    vc = vc.clone()
    kc[~used] = float("nan")
    vc[~used] = float("nan")
    return kc, vc


def _check(got, ref, lse_got=None, lse_ref=None):
    got = got.cpu().float()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err <= TOL, f"max abs err {err}"
    if lse_got is not None:
        a, b = lse_got.cpu(), lse_ref
        fin = torch.isfinite(b)
        assert torch.equal(torch.isfinite(a), fin)
        assert (a[fin] - b[fin]).abs().max().item() <= 1e-2 if fin.any() else True
    return err


@pytest.mark.parametrize("bs", [256, 16, 32, 64, 128])
@pytest.mark.parametrize("hkv", [8, 2])
def test_uniform_chunks_with_kvcache(pkg, cuda_dev, bs, hkv):
    """flash_attn_with_kvcache(q [B, Sq, Hq, D], ...) with prefixes of every
    kind: none, shorter than a tile, block-aligned, and long."""
    Sq, hq = 96, 16
    prefix = [0, 5, 64, 256, 700, 1000 - Sq]
    k_lens = [p + Sq for p in prefix]
    B = len(prefix)
    bt, nb = _tables(k_lens, bs, seed=bs + hkv)
    kc, vc = _pool(nb, bs, hkv, seed=1)
    kc, vc = _nan_tails(kc, vc, bt, k_lens, bs)  # nothing past a sequence's keys may reach the result
    g = torch.Generator().manual_seed(2)
    q = torch.randn(B, Sq, hq, 128, generator=g).to(torch.bfloat16)
    kl = torch.tensor(k_lens, dtype=torch.int32)
    out, lse = pkg.flash_attn_with_kvcache(q.to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev), cache_seqlens=kl.to(cuda_dev),
                                           block_table=bt.to(cuda_dev), causal=True, return_softmax_lse=True)
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    cu = torch.arange(B + 1, dtype=torch.int32) * Sq
    ref, ref_lse = opa.paged_chunk_prefill(q.view(B * Sq, hq, 128), kc, vc, bt, kl, cu, return_lse=True)
    assert out.shape == (B, Sq, hq, 128) and lse.shape == (B, hq, Sq)
    _check(out.view(B * Sq, hq, 128), ref, lse.permute(0, 2, 1).reshape(B * Sq, hq), ref_lse)


@pytest.mark.parametrize("bs", [256, 16])
def test_single_tile_chunks_rising_scores(pkg, cuda_dev, bs):
    """Three chunks of 448 queries over prefixes of 100-1100 keys: too few
    query-tile pairs to fill the SMs, so items are single tiles (both softmax
    warpgroups on one tile, S double buffered in TMEM) and some CTAs take
    two; keys scaled up along each sequence so that O is rescaled tile after
    tile; pool slots past each sequence's keys hold NaN. Values are scaled by
    1/4 for the same reason as in the contiguous rising-score test: peaked
    rows put whole value rows, rounded, into the bf16 output."""
    Sq, hq = 448, 16
    prefix = [100, 600, 1100]
    k_lens = [p + Sq for p in prefix]
    B = len(prefix)
    bt, nb = _tables(k_lens, bs, seed=70 + bs)
    kc, vc = _pool(nb, bs, 8, seed=71)
    kc, vc = kc.float(), vc.float() * 0.25
    for s, K in enumerate(k_lens):
        t = torch.arange(K)
        blk, slot = bt[s, t // bs].long(), t % bs
        kc[blk, slot] = kc[blk, slot] * (1 + 10.0 * t.float() / K).view(-1, 1, 1)
    kc, vc = _nan_tails(kc.to(torch.bfloat16), vc.to(torch.bfloat16), bt, k_lens, bs)
    g = torch.Generator().manual_seed(72)
    q = torch.randn(B, Sq, hq, 128, generator=g).to(torch.bfloat16)
    kl = torch.tensor(k_lens, dtype=torch.int32)
    out, lse = pkg.flash_attn_with_kvcache(q.to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev), cache_seqlens=kl.to(cuda_dev),
                                           block_table=bt.to(cuda_dev), causal=True, return_softmax_lse=True)
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    cu = torch.arange(B + 1, dtype=torch.int32) * Sq
    ref, ref_lse = opa.paged_chunk_prefill(q.view(B * Sq, hq, 128), kc, vc, bt, kl, cu, return_lse=True)
    _check(out.view(B * Sq, hq, 128), ref, lse.permute(0, 2, 1).reshape(B * Sq, hq), ref_lse)


@pytest.mark.parametrize("causal", [True, False])
def test_varlen_chunks_with_block_table(pkg, cuda_dev, causal):
    """flash_attn_varlen_func with a block_table: ragged chunk lengths (1 to
    300 tokens), ragged prefixes, one empty chunk, GQA group 2."""
    q_lens = [1, 17, 128, 0, 300, 64, 129, 2]
    prefix = [0, 900, 31, 40, 256, 1, 511, 2047]
    k_lens = [p + n for p, n in zip(prefix, q_lens)]
    bs = 256
    bt, nb = _tables(k_lens, bs, seed=5)
    kc, vc = _pool(nb, bs, 8, seed=6)
    kc, vc = _nan_tails(kc, vc, bt, k_lens, bs)
    cu_q = torch.zeros(len(q_lens) + 1, dtype=torch.int32)
    cu_q[1:] = torch.cumsum(torch.tensor(q_lens), 0)
    cu_k = torch.zeros(len(q_lens) + 1, dtype=torch.int32)
    cu_k[1:] = torch.cumsum(torch.tensor(k_lens), 0)
    T = int(cu_q[-1])
    q = torch.randn(T, 16, 128, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    d = cuda_dev
    out, lse = pkg.flash_attn_varlen_func(q.to(d), kc.to(d), vc.to(d), cu_q.to(d), cu_k.to(d), max(q_lens),
                                          max(k_lens), causal=causal, block_table=bt.to(d), return_softmax_lse=True)
    torch.cuda.synchronize()
    pkg.check_device_errors(d.index)
    ref, ref_lse = opa.paged_chunk_prefill(q, kc, vc, bt, torch.tensor(k_lens, dtype=torch.int32), cu_q,
                                           causal=causal, return_lse=True)
    _check(out, ref, lse.t(), ref_lse)


@pytest.mark.parametrize("hkv", [16, 4])
def test_gqa_groups(pkg, cuda_dev, hkv):
    Sq = 200
    k_lens = [Sq + 300, Sq]
    bt, nb = _tables(k_lens, 64, seed=hkv)
    kc, vc = _pool(nb, 64, hkv, seed=8)
    q = torch.randn(2, Sq, 16, 128, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    kl = torch.tensor(k_lens, dtype=torch.int32)
    d = cuda_dev
    out = pkg.flash_attn_with_kvcache(q.to(d), kc.to(d), vc.to(d), cache_seqlens=kl.to(d), block_table=bt.to(d),
                                      causal=True)
    torch.cuda.synchronize()
    ref = opa.paged_chunk_prefill(q.view(-1, 16, 128), kc, vc, bt, kl, torch.tensor([0, Sq, 2 * Sq], dtype=torch.int32))
    _check(out.view(-1, 16, 128), ref)


def test_rows_without_keys_are_zero(pkg, cuda_dev):
    """Fewer keys than chunk queries: the first rows see no key at all."""
    Sq = 80
    k_lens = [30, 0]
    bt, nb = _tables(k_lens, 256, seed=3)
    kc, vc = _pool(nb, 256, 8, seed=4)
    kc, vc = _nan_tails(kc, vc, bt, k_lens, 256)
    q = torch.randn(2, Sq, 16, 128, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    kl = torch.tensor(k_lens, dtype=torch.int32)
    d = cuda_dev
    out, lse = pkg.flash_attn_with_kvcache(q.to(d), kc.to(d), vc.to(d), cache_seqlens=kl.to(d), block_table=bt.to(d),
                                           causal=True, return_softmax_lse=True)
    torch.cuda.synchronize()
    pkg.check_device_errors(d.index)
    ref, ref_lse = opa.paged_chunk_prefill(q.view(-1, 16, 128), kc, vc, bt, kl,
                                           torch.tensor([0, Sq, 2 * Sq], dtype=torch.int32), return_lse=True)
    _check(out.view(-1, 16, 128), ref, lse.permute(0, 2, 1).reshape(-1, 16), ref_lse)
    assert torch.count_nonzero(out[0, :Sq - 30].float()) == 0 and torch.count_nonzero(out[1].float()) == 0


def test_bad_block_id_reported(pkg, cuda_dev):
    Sq = 64
    k_lens = [Sq + 256]
    bt, nb = _tables(k_lens, 256, seed=2)
    bt[0, 0] = nb + 5  # outside the pool
    kc, vc = _pool(nb, 256, 8, seed=2)
    q = torch.randn(1, Sq, 16, 128, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    d = cuda_dev
    out = pkg.flash_attn_with_kvcache(q.to(d), kc.to(d), vc.to(d), cache_seqlens=torch.tensor(k_lens, dtype=torch.int32,
                                      device=d), block_table=bt.to(d), causal=True)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()  # the bad block reads as zeros
    with pytest.raises(RuntimeError, match="block id"):
        pkg.check_device_errors(d.index)


def test_chunked_equals_whole_prefill_at_size(pkg, cuda_dev):
    """Size-independent property at full size: a 4096-token prompt prefilled
    in 512-token chunks over the paged cache gives the rows of one causal
    varlen prefill of the whole prompt (both on the GPU)."""
    d = cuda_dev
    L, C, bs = 4096, 512, 256
    g = torch.Generator(device=d).manual_seed(12)
    q = torch.randn(L, 16, 128, generator=g, device=d).to(torch.bfloat16)
    k = torch.randn(L, 8, 128, generator=g, device=d).to(torch.bfloat16)
    v = torch.randn(L, 8, 128, generator=g, device=d).to(torch.bfloat16)
    cu = torch.tensor([0, L], dtype=torch.int32, device=d)
    whole = pkg.flash_attn_varlen_func(q, k, v, cu, cu, L, L, causal=True)
    nblk = L // bs
    perm = (torch.randperm(nblk + 4, generator=torch.Generator().manual_seed(3))[:nblk] + 1).to(torch.int32)
    kc = torch.full((nblk + 6, bs, 8, 128), float("nan"), dtype=torch.bfloat16, device=d)
    vc = torch.full_like(kc, float("nan"))
    kc[perm.long().to(d)] = k.view(nblk, bs, 8, 128)
    vc[perm.long().to(d)] = v.view(nblk, bs, 8, 128)
    bt = perm.view(1, -1).to(d)
    outs = []
    for c0 in range(0, L, C):
        outs.append(pkg.flash_attn_with_kvcache(q[c0:c0 + C].view(1, C, 16, 128), kc, vc,
                                                cache_seqlens=torch.tensor([c0 + C], dtype=torch.int32, device=d),
                                                block_table=bt, causal=True))
    chunked = torch.cat([o.view(C, 16, 128) for o in outs])
    torch.cuda.synchronize()
    pkg.check_device_errors(d.index)
    err = (chunked.float() - whole.float()).abs().max().item()
    assert err <= TOL, err


def test_chunk_prefill_graph_replay(pkg, cuda_dev):
    """A fixed-size chunk is one captured graph: replays with new prefixes
    and new query values match the oracle."""
    d = cuda_dev
    B, Sq, bs = 4, 128, 256
    max_k = 1500
    bt, nb = _tables([max_k] * B, bs, seed=21)
    kc, vc = _pool(nb, bs, 8, seed=22)
    kcd, vcd, btd = kc.to(d), vc.to(d), bt.to(d)
    q_buf = torch.zeros(B, Sq, 16, 128, dtype=torch.bfloat16, device=d)
    kl_buf = torch.full((B,), Sq, dtype=torch.int32, device=d)
    pkg.flash_attn_with_kvcache(q_buf, kcd, vcd, cache_seqlens=kl_buf, block_table=btd, causal=True)  # warm-up
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = pkg.flash_attn_with_kvcache(q_buf, kcd, vcd, cache_seqlens=kl_buf, block_table=btd, causal=True)
    for it, prefix in enumerate(([0, 10, 300, 1000], [1372, 5, 128, 700])):
        q = torch.randn(B, Sq, 16, 128, generator=torch.Generator().manual_seed(30 + it)).to(torch.bfloat16)
        kl = torch.tensor([p + Sq for p in prefix], dtype=torch.int32)
        q_buf.copy_(q.to(d))
        kl_buf.copy_(kl.to(d))
        graph.replay()
        torch.cuda.synchronize()
        ref = opa.paged_chunk_prefill(q.view(-1, 16, 128), kc, vc, bt, kl, torch.arange(B + 1, dtype=torch.int32) * Sq)
        _check(out.view(-1, 16, 128), ref)
    pkg.check_device_errors(d.index)
    del graph
