"""The decode step's fused glue kernels (la_add_rms_norm, la_silu_mul)
against plain PyTorch fp32 references of the same ops. Tolerance: the
residual sum is bit-exact (one bf16 rounding of an fp32 sum); normalised and
activated outputs within one bf16 rounding (relative 2^-7) of the fp32
reference. The greedy-token argmax (la_argmax_rows) is index work: it must
equal torch.argmax exactly, ties, NaN and signed zeros included."""
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


@pytest.mark.parametrize("rows,cols,stride_pad,offset", [
    (128, 151936, 0, 0),    # the decode step's logits
    (3, 151936, 8, 0),      # padded rows
    (5, 1000, 0, 0),        # 1000 = 125 x 8: chunks only
    (4, 1003, 0, 0),        # 1003 = 125 x 8 + 3: tail elements
    (6, 777, 1, 0),         # rows not 16-byte aligned: element path
    (2, 4096, 0, 3),        # base not 16-byte aligned
    (1, 1, 0, 0),
])
def test_argmax_rows(pkg, cuda_dev, rows, cols, stride_pad, offset):
    from lean_infer_b200 import qwen3

    g = torch.Generator(device=cuda_dev).manual_seed(rows * 7 + cols)
    stride = cols + stride_pad
    buf = torch.randn(offset + rows * stride, generator=g, device=cuda_dev).to(torch.bfloat16)
    x = buf[offset:].view(rows, stride)[:, :cols]
    got = qwen3.argmax_rows(x)
    torch.cuda.synchronize()
    assert got.dtype == torch.int64 and torch.equal(got, x.argmax(-1))


def test_argmax_rows_ties_nan_zeros(pkg, cuda_dev):
    """Rows built so the answer depends on the tie and NaN rules."""
    from lean_infer_b200 import qwen3

    cols = 151936
    x = torch.full((10, cols), -3.0, device=cuda_dev, dtype=torch.bfloat16)
    x[0, [5000, 17, 90000]] = 2.0                  # tie: the first index
    x[1, [cols - 1, cols - 2]] = 1.0               # tie in the last chunk
    x[2] = float("-inf")                           # all -inf: index 0
    x[2, 123] = float("-inf")
    x[3, [70000, 4000]] = float("nan")             # NaN beats every number, first NaN
    x[3, 10] = float("inf")
    x[4] = 0.0                                     # signed zeros are equal
    x[4, :100] = -0.0
    x[5, [8, 9, 10, 11, 12, 13, 14, 15]] = 5.0     # a whole chunk of equal maxima
    x[6, 1] = float("inf")
    x[6, 1 + 8 * 512] = float("inf")               # same thread, later chunk
    x[7] = torch.arange(cols, device=cuda_dev).remainder(251).to(torch.bfloat16)  # many equal maxima
    x[8, cols - 3] = 7.0                           # max in the tail position of the row
    x[9, 0] = float("nan")
    got = qwen3.argmax_rows(x)
    torch.cuda.synchronize()
    assert torch.equal(got, x.argmax(-1)), (got.tolist(), x.argmax(-1).tolist())
