"""Host-side helpers of bench.py that feed its parity checks: the compact
copy of sampled rows the oracle reads, and the copy of a paged pool into a
pool of another block size (the 16-token-block step). CPU only."""
import torch

import bench
from oracle import paged_attention as opa


def _pool(nb, bs, g):
    return torch.randn(nb, bs, 2, 16, generator=g).to(torch.bfloat16)


def test_compact_rows_reads_what_the_full_pool_holds(pkg):
    from lean_infer_b200 import workloads as W

    g = torch.Generator().manual_seed(3)
    L = torch.tensor([1, 40, 17, 64, 33])
    bt, nb = W.deal_blocks(L, 16, 40, 5)
    kc, vc = _pool(nb, 16, g), _pool(nb, 16, g)
    q = torch.randn(5, 1, 4, 16, generator=g).to(torch.bfloat16)
    rows = [1, 3, 4]
    full = opa.paged_decode(q, kc, vc, bt, L.to(torch.int32))
    qr, kcr, vcr, btr, Lr = bench.compact_rows(q, kc, vc, bt, L.to(torch.int32), rows)
    assert kcr.shape[0] == sum(-(-int(L[r]) // 16) for r in rows)
    assert torch.equal(opa.paged_decode(qr, kcr, vcr, btr, Lr), full[rows])


def test_relayout_pool_keeps_every_cached_token(pkg):
    from lean_infer_b200 import workloads as W
    from lean_infer_b200.cache import BlockCache

    g = torch.Generator().manual_seed(4)
    L = torch.tensor([300, 5, 256, 511])
    src = BlockCache(2, 12, 128, 2, 16, "cpu")
    src.k.copy_(torch.randn(src.k.shape, generator=g).to(torch.bfloat16))
    src.v.copy_(torch.randn(src.v.shape, generator=g).to(torch.bfloat16))
    bt_s, _ = W.deal_blocks(L, 128, 12, 1)
    dst = BlockCache(2, 80, 16, 2, 16, "cpu")
    bt_d, _ = W.deal_blocks(L, 16, 80, 2)
    bench.relayout_pool(src, bt_s, dst, bt_d, L.to(torch.int32))
    q = torch.randn(4, 1, 4, 16, generator=g).to(torch.bfloat16)
    for layer in range(2):
        a = opa.paged_decode(q, src.k[layer], src.v[layer], bt_s, L.to(torch.int32))
        b = opa.paged_decode(q, dst.k[layer], dst.v[layer], bt_d, L.to(torch.int32))
        assert torch.equal(a, b)
