"""Fused QK-RMSNorm + RoPE + paged KV write (kernel a) and the plain paged
write. The cache write is checked bit-exact: against the oracle that fixes the
kernel's reduction order (everything bit-exact), against BlockCache.write fed
the same K/V (bit-exact), and against the reference's own outputs from the
golden fixtures (V bit-exact; normalised q/k within one bf16 ulp, because
torch sums the squares in a different order)."""
import numpy as np
import pytest
import torch

from oracle import pre_attention as opre

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _bf16(a):
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _ulp_diff(a, b):
    return (a.view(torch.int16).int() - b.view(torch.int16).int()).abs()


@pytest.mark.parametrize("name", ["pre_attention_decode.npz", "pre_attention_prefill.npz"])
def test_golden_fixture(pkg, cuda_dev, name):
    g = dict(np.load(GOLDEN / name))
    q, k, v = _bf16(g["q_raw"]), _bf16(g["k_raw"]), _bf16(g["v_raw"])
    qw, kw = _bf16(g["q_norm_w"]), _bf16(g["k_norm_w"])
    pos = torch.from_numpy(g["pos"]).long()
    bt = torch.from_numpy(g["block_table"]).int()
    q_len = int(g["q_len"])
    pool = torch.zeros_like(_bf16(g["pool_k_after"]))
    cos, sin = opre.rope_tables(2048, 128, 1e6)
    kc, vc = pool.clone().to(cuda_dev), pool.clone().to(cuda_dev)
    B = pos.shape[0]
    q_out = pkg.qk_norm_rope_paged_write(q.view(B, q_len, 16, 128).to(cuda_dev), k.view(B, q_len, 8, 128).to(cuda_dev),
                                         v.view(B, q_len, 8, 128).to(cuda_dev), qw.to(cuda_dev), kw.to(cuda_dev),
                                         cos.to(cuda_dev), sin.to(cuda_dev), pos.to(cuda_dev), bt.to(cuda_dev), kc, vc,
                                         eps=1e-6)
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    # bit-exact against the oracle in the kernel's order
    kr, vr = pool.clone(), pool.clone()
    q_ref, _ = opre.qk_norm_rope_paged_write(q, k, v, qw, kw, 1e-6, cos, sin, pos, bt, kr, vr, q_len=q_len)
    assert torch.equal(q_out.cpu(), q_ref)
    assert torch.equal(kc.cpu(), kr) and torch.equal(vc.cpu(), vr)
    # against the reference's own run: V exact, q/k within one ulp
    assert torch.equal(vc.cpu(), _bf16(g["pool_v_after"]))
    assert _ulp_diff(q_out.cpu(), _bf16(g["q_rope"])).max().item() <= 2
    assert _ulp_diff(kc.cpu(), _bf16(g["pool_k_after"])).max().item() <= 2


def _random_case(B, q_len, seed, bs=256, nb=600, max_pos=4096, varlen=None):
    g = torch.Generator().manual_seed(seed)
    if varlen is None:
        T = B * q_len
        pos = torch.randint(0, max_pos - q_len, (B,), generator=g)
        cu = None
        need = ((pos + q_len + bs - 1) // bs)
    else:
        lens = torch.tensor(varlen)
        cu = torch.zeros(B + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(lens, 0)
        T = int(cu[-1])
        pos = torch.randint(0, 500, (B,), generator=g)
        need = ((pos + lens + bs - 1) // bs)
    maxb = int(need.max())
    perm = torch.randperm(nb - 1, generator=g) + 1
    assert int(need.sum()) <= nb - 1
    bt = torch.zeros(B, maxb, dtype=torch.int32)
    o = 0
    for b in range(B):
        n = int(need[b])
        bt[b, :n] = perm[o:o + n].int()
        o += n
    q = (torch.randn(T, 16, 128, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(T, 8, 128, generator=g) * 2).to(torch.bfloat16)
    v = torch.randn(T, 8, 128, generator=g).to(torch.bfloat16)
    qw = (1 + 0.3 * torch.randn(128, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.3 * torch.randn(128, generator=g)).to(torch.bfloat16)
    pool = torch.randn(nb, bs, 8, 128, generator=g).to(torch.bfloat16)
    return q, k, v, qw, kw, pos, bt, cu, pool


@pytest.mark.parametrize("B,q_len,bs,max_pos", [(128, 1, 256, 1024), (3, 70, 16, 4096), (1, 1000, 256, 4096)])
def test_random_bit_exact(pkg, cuda_dev, B, q_len, bs, max_pos):
    q, k, v, qw, kw, pos, bt, cu, pool = _random_case(B, q_len, seed=B + q_len, bs=bs, nb=800, max_pos=max_pos)
    cos, sin = opre.rope_tables(4096, 128, 1e6)
    kc, vc = pool.clone().to(cuda_dev), pool.clone().to(cuda_dev)
    d = cuda_dev
    q_out = pkg.qk_norm_rope_paged_write(q.to(d), k.to(d), v.to(d), qw.to(d), kw.to(d), cos.to(d), sin.to(d),
                                         pos.to(d), bt.to(d), kc, vc)
    torch.cuda.synchronize()
    pkg.check_device_errors(d.index)
    kr, vr = pool.clone(), pool.clone()
    q_ref, _ = opre.qk_norm_rope_paged_write(q, k, v, qw, kw, 1e-6, cos, sin, pos, bt, kr, vr, q_len=q_len)
    assert torch.equal(q_out.cpu(), q_ref)
    assert torch.equal(kc.cpu(), kr)
    assert torch.equal(vc.cpu(), vr)


def test_varlen_bit_exact(pkg, cuda_dev):
    lens = [1, 37, 256, 257, 600, 5, 1024, 90]
    q, k, v, qw, kw, pos, bt, cu, pool = _random_case(len(lens), 0, seed=77, bs=256, nb=400, varlen=lens)
    cos, sin = opre.rope_tables(4096, 128, 1e6)
    kc, vc = pool.clone().to(cuda_dev), pool.clone().to(cuda_dev)
    d = cuda_dev
    q_out = pkg.qk_norm_rope_paged_write(q.to(d), k.to(d), v.to(d), qw.to(d), kw.to(d), cos.to(d), sin.to(d),
                                         pos.to(d), bt.to(d), kc, vc, cu_seqlens=cu.to(d))
    torch.cuda.synchronize()
    pkg.check_device_errors(d.index)
    kr, vr = pool.clone(), pool.clone()
    q_ref, _ = opre.qk_norm_rope_paged_write(q, k, v, qw, kw, 1e-6, cos, sin, pos, bt, kr, vr, cu_seqlens=cu)
    assert torch.equal(q_out.cpu(), q_ref)
    assert torch.equal(kc.cpu(), kr) and torch.equal(vc.cpu(), vr)


def test_paged_write_matches_block_cache_write(pkg, cuda_dev):
    """la_paged_kv_write == BlockCache.write (cache_manager.py:63-76), bit for
    bit, including idle rows that all write the trash block 0 at offset 0."""
    g = torch.Generator().manual_seed(3)
    B, q_len, bs, nb = 6, 3, 16, 40
    pos = torch.tensor([0, 14, 15, 100, 0, 0])
    bt = torch.zeros(B, 8, dtype=torch.int32)
    bt[:4] = (torch.randperm(nb - 1, generator=g)[:32] + 1).view(4, 8).int()
    k = torch.randn(B, 8, q_len, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, 8, q_len, 128, generator=g).to(torch.bfloat16)
    # idle rows 4, 5: identical content, so the duplicate writes are deterministic
    k[5], v[5] = k[4], v[4]
    pool = torch.randn(nb, bs, 8, 128, generator=g).to(torch.bfloat16)
    kr, vr = pool.clone(), pool.clone()
    opre.block_cache_write(kr, vr, bt, pos, k, v)
    cache = pkg.BlockCache(1, nb, bs, 8, 128, cuda_dev)
    cache.k[0].copy_(pool)
    cache.v[0].copy_(pool)
    cache.write(0, bt.to(cuda_dev), pos.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev))
    torch.cuda.synchronize()
    assert torch.equal(cache.k[0].cpu(), kr) and torch.equal(cache.v[0].cpu(), vr)


def test_rope_tables_on_device_match_reference_formula(pkg, cuda_dev):
    """The device tables equal build_rope's formula evaluated on the same
    device, and the CPU tables within one bf16 ulp."""
    cos_d, sin_d = pkg.rope_tables(40001, 128, 1e6, cuda_dev)
    pos = torch.tensor([0, 1, 255, 256, 1023, 8191, 32767, 40000], device=cuda_dev)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=cuda_dev).float() / 128))
    ang = pos[:, None].float() * inv
    emb = torch.cat((ang, ang), -1)
    assert torch.equal(cos_d[pos], emb.cos().to(torch.bfloat16)[:, :64])
    assert torch.equal(sin_d[pos], emb.sin().to(torch.bfloat16)[:, :64])
    # Against the reference's own build_rope run on the CPU (golden): CUDA's
    # pow/cos/sin and the CPU's differ by an fp32 ulp, which the angle scales
    # by the position, so only a loose bound holds across devices.
    g = dict(np.load(GOLDEN / "rope.npz"))
    gp = torch.from_numpy(g["pos"]).to(cuda_dev)
    assert (cos_d[gp].cpu().float() - _bf16(g["cos"])[:, :64].float()).abs().max().item() < 2e-2
    assert (sin_d[gp].cpu().float() - _bf16(g["sin"])[:, :64].float()).abs().max().item() < 2e-2


def test_bad_block_id_skips_write_and_reports(pkg, cuda_dev):
    q, k, v, qw, kw, pos, bt, cu, pool = _random_case(4, 1, seed=5, bs=256, nb=64)
    bt[2, :] = 5000
    cos, sin = opre.rope_tables(4096, 128, 1e6)
    d = cuda_dev
    kc, vc = pool.clone().to(d), pool.clone().to(d)
    pkg.qk_norm_rope_paged_write(q.to(d), k.to(d), v.to(d), qw.to(d), kw.to(d), cos.to(d), sin.to(d), pos.to(d),
                                 bt.to(d), kc, vc)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="block id"):
        pkg.check_device_errors(d.index)
    # the other rows were written, nothing else changed
    kr, vr = pool.clone(), pool.clone()
    keep = torch.tensor([0, 1, 3])
    opre.qk_norm_rope_paged_write(q[keep], k[keep], v[keep], qw, kw, 1e-6, cos, sin, pos[keep], bt[keep], kr, vr,
                                  q_len=1)
    assert torch.equal(kc.cpu(), kr) and torch.equal(vc.cpu(), vr)


@pytest.mark.parametrize("q_len", [1, 33])
def test_idle_rows_write_nothing(pkg, cuda_dev, q_len):
    """A negative start position marks an idle row: its cache slots stay
    untouched (no trash block needed), its q / k outputs are zeros, no error."""
    B = 12
    q, k, v, qw, kw, pos, bt, cu, pool = _random_case(B, q_len, seed=5 + q_len, bs=256, nb=400, max_pos=4096)
    pos = pos.clone()
    pos[1::3] = -1
    cos, sin = opre.rope_tables(4096, 128, 1e6)
    kc, vc = pool.clone().to(cuda_dev), pool.clone().to(cuda_dev)
    d = cuda_dev
    k_out = torch.empty_like(k).to(d)
    q_out = pkg.qk_norm_rope_paged_write(q.to(d), k.to(d), v.to(d), qw.to(d), kw.to(d), cos.to(d), sin.to(d),
                                         pos.to(d), bt.to(d), kc, vc, k_out=k_out)
    torch.cuda.synchronize()
    pkg.check_device_errors(d.index)  # idle rows raise nothing
    kr, vr = pool.clone(), pool.clone()
    q_ref, k_ref = opre.qk_norm_rope_paged_write(q, k, v, qw, kw, 1e-6, cos, sin, pos, bt, kr, vr, q_len=q_len)
    assert torch.equal(q_out.cpu(), q_ref) and torch.equal(k_out.cpu(), k_ref)
    assert torch.equal(kc.cpu(), kr) and torch.equal(vc.cpu(), vr)
    idle_tok = (pos < 0).repeat_interleave(q_len)
    assert torch.count_nonzero(q_out.cpu()[idle_tok]) == 0
