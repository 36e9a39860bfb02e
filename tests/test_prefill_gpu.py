"""Causal varlen prefill (kernel c, tcgen05/TMEM) against the fp32 CPU oracle
and the reference's own SDPA output (golden fixture).

Tolerance: max |out - oracle| <= 2e-2 on bf16 outputs; lse within 1e-2."""
import numpy as np
import pytest
import torch

from oracle import paged_attention as opa

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _case(lengths, hq=16, hkv=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    lens = torch.tensor(lengths, dtype=torch.int64)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    T = int(cu[-1])
    q = torch.randn(T, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(T, hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(T, hkv, 128, generator=g).to(torch.bfloat16)
    return q, k, v, cu, int(lens.max()) if len(lengths) else 0


def run(pkg, dev, lengths, hq=16, hkv=8, seed=0, causal=True, lse=False, key_ramp=0.0, v_scale=1.0):
    q, k, v, cu, mx = _case(lengths, hq, hkv, seed)
    if v_scale != 1.0:
        v = (v.float() * v_scale).to(torch.bfloat16)
    if key_ramp:  # keys scaled up along each sequence: the running row max keeps rising
        pos = torch.cat([torch.arange(n, dtype=torch.float32) / max(n, 1) for n in lengths])
        k = (k.float() * (1 + key_ramp * pos).view(-1, 1, 1)).to(torch.bfloat16)
    cud = cu.to(dev)
    res = pkg.flash_attn_varlen_func(q.to(dev), k.to(dev), v.to(dev), cud, cud, mx, mx, causal=causal,
                                     return_softmax_lse=lse)
    out, lse_d = res if lse else (res, None)
    torch.cuda.synchronize()
    pkg.check_device_errors(dev.index)
    if causal:
        ref = opa.varlen_causal_prefill(q, k, v, cu, return_lse=lse)
    else:
        ref = _noncausal(q, k, v, cu)
    ref, ref_lse = ref if lse else (ref, None)
    got = out.cpu().float()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err <= TOL, f"max abs err {err}"
    if lse:
        assert (lse_d.cpu().t() - ref_lse).abs().max().item() <= 1e-2
    return err


def _noncausal(q, k, v, cu):
    out = torch.zeros(q.shape, dtype=torch.float32)
    for s in range(cu.numel() - 1):
        a, b = int(cu[s]), int(cu[s + 1])
        if b > a:
            o = torch.nn.functional.scaled_dot_product_attention(
                q[a:b].float().transpose(0, 1)[None], k[a:b].float().transpose(0, 1)[None],
                v[a:b].float().transpose(0, 1)[None], enable_gqa=True)
            out[a:b] = o[0].transpose(0, 1)
    return out


def test_golden_reference_sdpa(pkg, cuda_dev):
    """The reference's own fp32 SDPA prefill (model.py:56-57), L=80."""
    g = dict(np.load(GOLDEN / "attention_prefill.npz"))
    q = torch.from_numpy(g["q"]).transpose(0, 1).contiguous().to(torch.bfloat16)
    k = torch.from_numpy(g["k"]).transpose(0, 1).contiguous().to(torch.bfloat16)
    v = torch.from_numpy(g["v"]).transpose(0, 1).contiguous().to(torch.bfloat16)
    L = q.shape[0]
    cu = torch.tensor([0, L], dtype=torch.int32, device=cuda_dev)
    out = pkg.flash_attn_varlen_func(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), cu, cu, L, L, causal=True)
    err = (out.cpu().float() - torch.from_numpy(g["o"]).transpose(0, 1)).abs().max().item()
    assert err <= TOL, err


def test_config_b16_packed(pkg, cuda_dev):
    """16 packed prompts, lengths U[512,1024]."""
    from lean_infer_b200 import workloads as W

    L = W.seq_lengths(16, 512, 1024, 3).tolist()
    run(pkg, cuda_dev, L, seed=1, lse=True)


def test_config_b1(pkg, cuda_dev):
    run(pkg, cuda_dev, [777], seed=2)


@pytest.mark.parametrize("n", [3, 16])
def test_rising_scores(pkg, cuda_dev, n):
    """Scores that grow along the keys, so O is rescaled tile after tile.
    Three prompts of 700 tokens leave too few query-tile pairs to fill the
    SMs: items are single tiles (both softmax warpgroups on one tile, S
    double buffered in TMEM) and most CTAs take two of them; sixteen
    prompts run as pairs. Peaked softmax rows make each output close to one
    value row, and with the running max raised only past +8 (log2) the
    dominant P is a rounded bf16 value rather than exactly 1 (about 0.013 on
    unit-variance values, by a CPU emulation of the algorithm), on top of
    the bf16 rounding of the output (half an ulp is 2^-8 |out|): the values
    are scaled by 1/4 to keep both well inside the absolute tolerance. A
    missing or misplaced rescale would still miss by the size of the output."""
    run(pkg, cuda_dev, [700] * n, seed=40 + n, lse=True, key_ramp=10.0, v_scale=0.25)


@pytest.mark.parametrize("L", [1, 2, 63, 64, 65, 127, 128, 129, 255, 256, 1024, 1100])
def test_lengths(pkg, cuda_dev, L):
    run(pkg, cuda_dev, [L], seed=L)


def test_ragged_with_empty(pkg, cuda_dev):
    run(pkg, cuda_dev, [5, 0, 300, 1, 0, 129, 64], seed=9, lse=True)


@pytest.mark.parametrize("group", [1, 4, 8])
def test_group_sizes(pkg, cuda_dev, group):
    run(pkg, cuda_dev, [100, 333, 17], hq=4 * group, hkv=4, seed=20 + group)


def test_noncausal(pkg, cuda_dev):
    run(pkg, cuda_dev, [200, 77, 300], seed=31, causal=False)


def test_sdpa_drop_in(pkg, cuda_dev):
    """The call-site form: q [B, Hq, L, D], k/v [B, Hkv, L, D]."""
    g = torch.Generator().manual_seed(4)
    B, L = 2, 300
    q = torch.randn(B, L, 16, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(B, L, 8, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    v = torch.randn(B, L, 8, 128, generator=g).to(torch.bfloat16).transpose(1, 2)
    out = pkg.scaled_dot_product_attention(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), is_causal=True,
                                           enable_gqa=True)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True,
                                                           enable_gqa=True)
    assert out.shape == q.shape
    assert (out.cpu().float() - ref).abs().max().item() <= TOL


def test_max_seqlen_too_small_reported(pkg, cuda_dev):
    q, k, v, cu, mx = _case([300, 40])
    pkg.flash_attn_varlen_func(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), cu.to(cuda_dev), cu.to(cuda_dev),
                               100, 100, causal=True)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="longer"):
        pkg.check_device_errors(cuda_dev.index)


def test_matches_flash_attn_varlen(pkg, cuda_dev):
    """Against flash-attn 2.8.3's varlen kernel on the same packed prompts."""
    fa = pytest.importorskip("flash_attn")
    from lean_infer_b200 import workloads as W

    w = W.prefill_batch(16, 512, 1024, seed=3, device=cuda_dev)
    mx = int(w.lengths.max())
    try:
        ref = fa.flash_attn_varlen_func(w.q, w.k, w.v, w.cu_seqlens, w.cu_seqlens, mx, mx, causal=True)
    except RuntimeError as e:
        pytest.skip(f"flash_attn_varlen_func does not run here: {e}")
    out = pkg.flash_attn_varlen_func(w.q, w.k, w.v, w.cu_seqlens, w.cu_seqlens, mx, mx, causal=True)
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max().item() <= TOL


# One prompt (the reference's own prefill shape, B=1): single-tile items.
@pytest.mark.parametrize("L", [300, 525, 700, 1024, 1500, 2000])
def test_single_prompt(pkg, cuda_dev, L):
    run(pkg, cuda_dev, [L], seed=L, lse=True)


def test_sdpa_single_prompt_strided_views(pkg, cuda_dev):
    """The SDPA drop-in at B=1 passes the [1, H, L, D] tensors' strides to the
    kernel (no copies); results match the oracle."""
    L = 640
    q, k, v, cu, _ = _case([L], seed=21)
    qd = q.to(cuda_dev).transpose(0, 1)[None]  # [1, Hq, L, D] views of [L, Hq, D]
    kd = k.to(cuda_dev).transpose(0, 1)[None]
    vd = v.to(cuda_dev).transpose(0, 1)[None]
    out = pkg.scaled_dot_product_attention(qd, kd, vd, is_causal=True, enable_gqa=True)
    torch.cuda.synchronize()
    ref = opa.varlen_causal_prefill(q, k, v, cu)
    assert (out[0].transpose(0, 1).cpu().float() - ref).abs().max().item() <= TOL


def test_cu_seqlens_rewritten_on_the_stream_between_calls(pkg, cuda_dev):
    """The one-prompt kernel instance reads cu_seqlens before its dependency
    wait (to walk to its first item early) and checks them again after it.
    Here the same cu_seqlens tensor is overwritten on the stream right before
    each call, with different lengths each time, and no synchronisation in
    between: every call must see its own lengths (against the oracle)."""
    lens_list = [[300, 200], [100, 700], [640], [2, 511, 64], [129, 127]]
    cases = [_case(l, seed=40 + i) for i, l in enumerate(lens_list)]
    T = max(int(c[3][-1]) for c in cases)
    q_d = torch.zeros(T, 16, 128, dtype=torch.bfloat16, device=cuda_dev)
    k_d = torch.zeros(T, 8, 128, dtype=torch.bfloat16, device=cuda_dev)
    v_d = torch.zeros(T, 8, 128, dtype=torch.bfloat16, device=cuda_dev)
    cu_d = torch.zeros(4, dtype=torch.int32, device=cuda_dev)
    staged = [(c[0].to(cuda_dev), c[1].to(cuda_dev), c[2].to(cuda_dev), c[3].to(cuda_dev)) for c in cases]
    outs = []
    torch.cuda.synchronize()
    for (q, k, v, cu), (_, _, _, cu_h, mx) in zip(staged, cases):
        n = q.shape[0]
        q_d[:n].copy_(q)
        k_d[:n].copy_(k)
        v_d[:n].copy_(v)
        cu_view = cu_d[: cu.numel()]
        cu_view.copy_(cu)  # a device copy on the stream, just before the kernel
        out = pkg.flash_attn_varlen_func(q_d[:n], k_d[:n], v_d[:n], cu_view, cu_view, mx, mx, causal=True)
        outs.append(out[:n].clone())
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    for (q, k, v, cu, _), out in zip(cases, outs):
        ref = opa.varlen_causal_prefill(q, k, v, cu)
        assert (out.cpu().float() - ref).abs().max().item() <= TOL
