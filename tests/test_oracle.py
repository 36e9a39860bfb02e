"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py). No GPU needed."""
import numpy as np
import pytest
import torch

from oracle import paged_attention as opa
from oracle import pre_attention as opre

from conftest import GOLDEN


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _load(name):
    return dict(np.load(GOLDEN / name))


def test_rope_matches_build_rope():
    g = _load("rope.npz")
    pos = torch.from_numpy(g["pos"])
    cos, sin = opre.build_rope(pos, 1, 128, 1e6)
    assert torch.equal(cos[:, 0, 0], _bf16(g["cos"]))
    assert torch.equal(sin[:, 0, 0], _bf16(g["sin"]))
    # the absolute-position tables hold the same values (first half)
    ct, st = opre.rope_tables(40001, 128, 1e6)
    assert torch.equal(ct[pos], _bf16(g["cos"])[:, :64])
    assert torch.equal(st[pos], _bf16(g["sin"])[:, :64])
    assert torch.equal(_bf16(g["cos"])[:, 64:], _bf16(g["cos"])[:, :64])


@pytest.mark.parametrize("name", ["pre_attention_decode.npz", "pre_attention_prefill.npz"])
def test_pre_attention_reference_norm_exact(name):
    """Oracle with torch's rms_norm reproduces the reference bit for bit:
    q after norm+rope, k after norm+rope, and the pool after BlockCache.write."""
    g = _load(name)
    q, k, v = _bf16(g["q_raw"]), _bf16(g["k_raw"]), _bf16(g["v_raw"])
    pos = torch.from_numpy(g["pos"]).long()
    bt = torch.from_numpy(g["block_table"]).int()
    q_len = int(g["q_len"])
    pk = torch.zeros_like(_bf16(g["pool_k_after"]))
    pv = torch.zeros_like(pk)
    cos, sin = opre.rope_tables(2048, 128, 1e6)
    q_out, k_out = opre.qk_norm_rope_paged_write(q, k, v, _bf16(g["q_norm_w"]), _bf16(g["k_norm_w"]), 1e-6, cos,
                                                 sin, pos, bt, pk, pv, q_len=q_len, norm="reference")
    assert torch.equal(q_out, _bf16(g["q_rope"]))
    assert torch.equal(k_out, _bf16(g["k_rope"]))
    assert torch.equal(pk, _bf16(g["pool_k_after"]))
    assert torch.equal(pv, _bf16(g["pool_v_after"]))


@pytest.mark.parametrize("name", ["pre_attention_decode.npz", "pre_attention_prefill.npz"])
def test_pre_attention_kernel_order_within_one_ulp(name):
    """The kernel's fixed reduction order differs from torch's by at most one
    bf16 ulp, in very few elements."""
    g = _load(name)
    q, k, v = _bf16(g["q_raw"]), _bf16(g["k_raw"]), _bf16(g["v_raw"])
    pos = torch.from_numpy(g["pos"]).long()
    bt = torch.from_numpy(g["block_table"]).int()
    pk = torch.zeros_like(_bf16(g["pool_k_after"]))
    pv = torch.zeros_like(pk)
    cos, sin = opre.rope_tables(2048, 128, 1e6)
    q_out, k_out = opre.qk_norm_rope_paged_write(q, k, v, _bf16(g["q_norm_w"]), _bf16(g["k_norm_w"]), 1e-6, cos,
                                                 sin, pos, bt, pk, pv, q_len=int(g["q_len"]), norm="kernel")
    for got, want in ((q_out, _bf16(g["q_rope"])), (k_out, _bf16(g["k_rope"]))):
        diff = got.view(torch.int16).int() - want.view(torch.int16).int()
        assert diff.abs().max().item() <= 2  # <=1 ulp after rope's three roundings (sign-magnitude)
        assert (diff != 0).float().mean().item() < 1e-3
    assert torch.equal(pv, _bf16(g["pool_v_after"]))


def test_kernel_order_norm_vs_torch_statistics():
    """Over many random rows, the fixed-order norm equals torch's in all but a
    few elements per million, each off by one ulp."""
    gen = torch.Generator().manual_seed(1)
    x = (torch.randn(4096, 128, generator=gen) * 3).to(torch.bfloat16)
    w = (1 + 0.5 * torch.randn(128, generator=gen)).to(torch.bfloat16)
    a = opre.rms_norm_kernel_order(x, w, 1e-6)
    b = opre.rms_norm_reference(x, w, 1e-6)
    diff = (a.view(torch.int16).int() - b.view(torch.int16).int()).abs()
    assert diff.max().item() <= 1
    assert (diff != 0).float().mean().item() < 1e-4


def test_block_cache_write_matches_reference():
    g = _load("pre_attention_decode.npz")
    B = g["pos"].shape[0]
    k = _bf16(g["k_rope"]).view(B, 1, 8, 128).transpose(1, 2)  # [B, Hkv, 1, D]
    v = _bf16(g["v_raw"]).view(B, 1, 8, 128).transpose(1, 2)
    pk = torch.zeros_like(_bf16(g["pool_k_after"]))
    pv = torch.zeros_like(pk)
    opre.block_cache_write(pk, pv, torch.from_numpy(g["block_table"]).int(), torch.from_numpy(g["pos"]).long(), k, v)
    assert torch.equal(pk, _bf16(g["pool_k_after"]))
    assert torch.equal(pv, _bf16(g["pool_v_after"]))


def test_allocator_fifo_and_trash_block():
    a = opre.BlockAllocator(6)
    assert a.allocate(2) == [1, 2]
    a.release([1])
    assert a.allocate(3) == [3, 4, 5]
    assert a.allocate(1) == [1]
    with pytest.raises(AssertionError):
        a.allocate(1)


def test_prefill_oracle_matches_reference_sdpa():
    g = _load("attention_prefill.npz")
    q = torch.from_numpy(g["q"]).transpose(0, 1)  # [L, Hq, D]
    k = torch.from_numpy(g["k"]).transpose(0, 1)
    v = torch.from_numpy(g["v"]).transpose(0, 1)
    L = q.shape[0]
    out = opa.varlen_causal_prefill(q, k, v, torch.tensor([0, L], dtype=torch.int32))
    torch.testing.assert_close(out, torch.from_numpy(g["o"]).transpose(0, 1), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("block_size", [16, 256])
def test_decode_oracle_pinned_by_reference_prefill(block_size):
    """A decode query at position t over keys 0..t (paged, permuted blocks)
    equals row t of the reference's causal prefill output."""
    g = _load("attention_prefill.npz")
    q = torch.from_numpy(g["q"]).transpose(0, 1)  # [L, Hq, D]
    k = torch.from_numpy(g["k"]).transpose(0, 1)
    v = torch.from_numpy(g["v"]).transpose(0, 1)
    o = torch.from_numpy(g["o"]).transpose(0, 1)
    L = q.shape[0]
    nblk = -(-L // block_size)
    NB = nblk + 3
    perm = torch.randperm(NB - 1, generator=torch.Generator().manual_seed(5))[:nblk] + 1
    kc = torch.full((NB, block_size, 8, 128), float("nan"))
    vc = torch.full((NB, block_size, 8, 128), float("nan"))
    for i in range(nblk):
        n = min(block_size, L - i * block_size)
        kc[perm[i], :n] = k[i * block_size: i * block_size + n]
        vc[perm[i], :n] = v[i * block_size: i * block_size + n]
    ts = torch.arange(L)
    B = L
    qd = q.view(L, 1, 16, 128)
    bt = perm.view(1, -1).expand(B, -1).int()
    out, lse = opa.paged_decode(qd, kc, vc, bt, (ts + 1).int(), return_lse=True)
    torch.testing.assert_close(out[:, 0], o, rtol=1e-5, atol=1e-5)
    _, lse_p = opa.varlen_causal_prefill(q, k, v, torch.tensor([0, L], dtype=torch.int32), return_lse=True)
    torch.testing.assert_close(lse, lse_p, rtol=1e-5, atol=1e-5)
    # padded batch form used as the CPU baseline agrees (NaN-filled tails never reach it)
    out_p = opa.paged_decode_padded(qd, kc.nan_to_num(), vc.nan_to_num(), bt, (ts + 1).int())
    torch.testing.assert_close(out_p, out, rtol=1e-5, atol=1e-5)


def test_decode_oracle_empty_rows_zero():
    kc = torch.randn(4, 16, 8, 128)
    out = opa.paged_decode(torch.randn(2, 1, 16, 128), kc, kc, torch.ones(2, 1, dtype=torch.int32),
                           torch.tensor([0, 5], dtype=torch.int32))
    assert torch.count_nonzero(out[0]) == 0
    assert torch.count_nonzero(out[1]) > 0


@pytest.mark.parametrize("block_size,chunk", [(16, 32), (16, 7), (256, 80), (64, 33)])
def test_chunk_prefill_oracle_pinned_by_reference_prefill(block_size, chunk):
    """A prompt processed in chunks over the paged cache (each chunk's keys
    already in the cache, bottom-right causal) gives the rows of the
    reference's full causal prefill; NaN-filled pool slots past the written
    keys never reach the result."""
    g = _load("attention_prefill.npz")
    q = torch.from_numpy(g["q"]).transpose(0, 1)
    k = torch.from_numpy(g["k"]).transpose(0, 1)
    v = torch.from_numpy(g["v"]).transpose(0, 1)
    o = torch.from_numpy(g["o"]).transpose(0, 1)
    L = q.shape[0]
    nblk = -(-L // block_size)
    NB = nblk + 2
    perm = torch.randperm(NB - 1, generator=torch.Generator().manual_seed(9))[:nblk] + 1
    kc = torch.full((NB, block_size, 8, 128), float("nan"))
    vc = torch.full((NB, block_size, 8, 128), float("nan"))
    for t in range(L):
        kc[perm[t // block_size], t % block_size] = k[t]
        vc[perm[t // block_size], t % block_size] = v[t]
    bt = perm.view(1, -1).int()
    # all chunks of the prompt packed as one call: sequence c = chunk c with its own prefix
    starts = list(range(0, L, chunk))
    ends = [min(L, s + chunk) for s in starts]
    cu = torch.tensor([0] + list(np.cumsum([e - s for s, e in zip(starts, ends)])), dtype=torch.int32)
    out, lse = opa.paged_chunk_prefill(q, kc, vc, bt.expand(len(starts), -1), torch.tensor(ends, dtype=torch.int32),
                                       cu, return_lse=True)
    torch.testing.assert_close(out, o, rtol=1e-5, atol=1e-5)
    _, lse_p = opa.varlen_causal_prefill(q, k, v, torch.tensor([0, L], dtype=torch.int32), return_lse=True)
    torch.testing.assert_close(lse, lse_p, rtol=1e-5, atol=1e-5)


def test_chunk_prefill_oracle_rows_without_keys():
    """Fewer keys than queries: the first n-K rows see no key (zeros, lse -inf)."""
    kc = torch.randn(4, 16, 8, 128)
    q = torch.randn(6, 16, 128)
    out, lse = opa.paged_chunk_prefill(q, kc, kc, torch.tensor([[1, 2]], dtype=torch.int32),
                                       torch.tensor([4], dtype=torch.int32), torch.tensor([0, 6], dtype=torch.int32),
                                       return_lse=True)
    assert torch.count_nonzero(out[:2]) == 0 and torch.isinf(lse[:2]).all()
    assert torch.isfinite(out[2:]).all() and torch.count_nonzero(out[2]) > 0


def test_full_step_port_matches_reference_model():
    """oracle/qwen3_step.py (the CPU baseline and the model tests' oracle)
    against the reference's own Qwen3ForCausalLM on the same seeded fp32
    weights (tests/golden/model_step.npz): two prompts prefilled one at a
    time, then one decode step of both rows. Both sides are fp32 on the CPU
    and differ only in summation order, so the bound is tight: 1e-4 relative
    to the largest logit, identical argmax, and the pool rows the same to 1e-5."""
    from oracle.qwen3_step import CpuQwen3Decode, seeded_weights

    g = _load("model_step.npz")
    c = dict(layers=2, hidden=1024, heads=16, kv_heads=8, head_dim=128, inter=3072, vocab=2048, eps=1e-6, theta=1e6)
    w = seeded_weights(c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["inter"], c["vocab"], 21)
    port = CpuQwen3Decode.from_weights(w, c, 8, 256)
    bt = torch.from_numpy(g["block_table"]).int()
    lens = [int(x) for x in g["lens"]]
    for i, L in enumerate(lens):
        ids = torch.from_numpy(g[f"prompt{i}"]).long().view(1, L)
        lg = port.forward(ids, torch.zeros(1, dtype=torch.long), bt[i:i + 1], None)[0, -3:]
        want = torch.from_numpy(g[f"prefill_logits{i}"])
        assert (lg - want).abs().max().item() <= 1e-4 * want.abs().max().item()
        assert torch.equal(lg.argmax(-1), want.argmax(-1))
    ids = torch.from_numpy(g["decode_ids"]).long()
    pos = torch.tensor(lens, dtype=torch.long)
    lg = port.forward(ids, pos, bt, (pos + 1).to(torch.int32))[:, 0]
    want = torch.from_numpy(g["decode_logits"])
    assert (lg - want).abs().max().item() <= 1e-4 * want.abs().max().item()
    assert torch.equal(lg.argmax(-1), want.argmax(-1))
    for j, (i, t) in enumerate(g["pool_positions"]):
        blk, off = int(bt[i, t // 256]), int(t % 256)
        for layer in range(2):
            assert (port.k_pools[layer, blk, off] - torch.from_numpy(g["pool_k"][j, layer])).abs().max() <= 1e-5
            assert (port.v_pools[layer, blk, off] - torch.from_numpy(g["pool_v"][j, layer])).abs().max() <= 1e-5
