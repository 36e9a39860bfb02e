"""The decode step's fused glue kernels (la_add_rms_norm, la_silu_mul)
against plain PyTorch fp32 references of the same ops. Tolerance: the
residual sum is bit-exact (one bf16 rounding of an fp32 sum); normalised and
activated outputs within one bf16 rounding (relative 2^-7) of the fp32
reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu
ULP = 2.0 ** -7


def _close(got, ref):
    got, ref = got.float(), ref.float()
    return bool(((got - ref).abs() <= ULP * ref.abs() + 1e-6).all())


@pytest.mark.parametrize("T,n", [(128, 1024), (1000, 1024), (3, 4096), (1, 8)])
def test_add_rms_norm(pkg, cuda_dev, T, n):
    from lean_infer_b200 import qwen3

    g = torch.Generator(device=cuda_dev).manual_seed(T + n)
    h = torch.randn(T, n, generator=g, device=cuda_dev).to(torch.bfloat16)
    a = (3 * torch.randn(T, n, generator=g, device=cuda_dev)).to(torch.bfloat16)
    w = (1 + 0.2 * torch.randn(n, generator=g, device=cuda_dev)).to(torch.bfloat16)
    hs_ref = (h.float() + a.float()).to(torch.bfloat16)
    x_ref = hs_ref.float() * torch.rsqrt(hs_ref.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    h_in = h.clone()
    h_out, x = qwen3.add_rms_norm(h_in, a, w, 1e-6)
    torch.cuda.synchronize()
    assert h_out.data_ptr() == h_in.data_ptr() and torch.equal(h_out, hs_ref)  # in place, bit-exact
    assert _close(x, x_ref)
    # without an addend: plain RMSNorm, h untouched
    h2 = h.clone()
    same, x2 = qwen3.add_rms_norm(h2, None, w, 1e-6)
    x2_ref = h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    torch.cuda.synchronize()
    assert torch.equal(same, h) and _close(x2, x2_ref)
    # matches torch's own bf16 rms_norm to within one rounding
    assert _close(x2, torch.nn.functional.rms_norm(h, (n,), w, 1e-6).float())


@pytest.mark.parametrize("T,n", [(128, 3072), (7, 8), (1000, 3072)])
def test_silu_mul(pkg, cuda_dev, T, n):
    from lean_infer_b200 import qwen3

    g = torch.Generator(device=cuda_dev).manual_seed(T * 7 + n)
    gu = (2 * torch.randn(T, 2 * n, generator=g, device=cuda_dev)).to(torch.bfloat16)
    out = qwen3.silu_mul(gu, n)
    ref = torch.nn.functional.silu(gu[:, :n].float()) * gu[:, n:].float()
    torch.cuda.synchronize()
    assert out.shape == (T, n) and _close(out, ref)
