"""la_o_proj_gathered, the o_proj GEMM of the KV-head-sharded partition
(leaninfer/qwen3/model.py:68-69), through the C ABI on one GPU.

With world = 1 it is a plain bf16 GEMM (fp32 accumulation on tcgen05): it
must match torch's fp32 product of the same bf16 operands to one bf16
rounding of the output. With world = 2 on one GPU the second rank's columns
are guarded by its epoch word, which the test publishes by hand (the GEMM
then runs) or never publishes (the bounded wait runs out, the error word
says so and the context stays usable). The multi-GPU form is in
tests/test_sharding_gpu.py."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(lib, a, w, out, signals, world, rank, err, dev):
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    return lib.la_o_proj_gathered(ctypes.c_void_p(a.data_ptr()), a.stride(0), ctypes.c_void_p(w.data_ptr()),
                                  w.stride(0), ctypes.c_void_p(out.data_ptr()), out.stride(0), a.shape[0],
                                  w.shape[0], a.shape[1], ctypes.c_void_p(signals.data_ptr()), world, rank,
                                  ctypes.c_void_p(err.data_ptr()), stream)


def _check(out, a, w):
    ref = a.float() @ w.float().T
    # one bf16 rounding of the output (2^-8 relative) plus fp32 order effects
    tol = 2 ** -8 * ref.abs() + 1e-5 * ref.abs().max()
    assert torch.all((out.float() - ref).abs() <= tol + 1e-6), (out.float() - ref).abs().max().item()


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 2048), (128, 1024, 2048), (1, 1024, 2048), (300, 512, 1024),
                                   (77, 2048, 256), (1000, 96, 128)])
def test_o_proj_plain_gemm(pkg, cuda_dev, m, n, k):
    from lean_infer_b200 import _lib
    from lean_infer_b200 import flash_attn_interface as fai

    lib = _lib.load()
    assert lib.la_init(cuda_dev.index) == 0
    g = torch.Generator(device=cuda_dev).manual_seed(m + n + k)
    a = (0.3 * torch.randn(m, k, generator=g, device=cuda_dev)).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=cuda_dev) / k ** 0.5).to(torch.bfloat16)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
    signals = torch.zeros(8, dtype=torch.int32, device=cuda_dev)
    err = fai.error_word(cuda_dev.index)
    assert _call(lib, a, w, out, signals, 1, 0, err, cuda_dev) == 0
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    _check(out, a, w)


def test_o_proj_strided_rows(pkg, cuda_dev):
    """Rows of the gather slot and of the output with padding between them."""
    from lean_infer_b200 import _lib
    from lean_infer_b200 import flash_attn_interface as fai

    lib = _lib.load()
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    base = torch.randn(200, 2048 + 64, generator=g, device=cuda_dev).to(torch.bfloat16)
    a = base[:, :2048]
    w = (torch.randn(1024, 2048, generator=g, device=cuda_dev) / 45).to(torch.bfloat16)
    obuf = torch.zeros(200, 1024 + 32, dtype=torch.bfloat16, device=cuda_dev)
    out = obuf[:, :1024]
    signals = torch.zeros(8, dtype=torch.int32, device=cuda_dev)
    assert _call(lib, a, w, out, signals, 1, 0, fai.error_word(cuda_dev.index), cuda_dev) == 0
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    _check(out, a, w)
    assert torch.equal(obuf[:, 1024:], torch.zeros_like(obuf[:, 1024:]))


def test_o_proj_waits_for_the_peer_epoch(pkg, cuda_dev):
    """world = 2: rank 1's half of the columns is read only once rank 1's
    epoch word reaches this rank's own epoch."""
    import time

    from lean_infer_b200 import _lib
    from lean_infer_b200 import flash_attn_interface as fai

    lib = _lib.load()
    g = torch.Generator(device=cuda_dev).manual_seed(4)
    a = torch.randn(256, 2048, generator=g, device=cuda_dev).to(torch.bfloat16)
    w = (torch.randn(1024, 2048, generator=g, device=cuda_dev) / 45).to(torch.bfloat16)
    out = torch.zeros(256, 1024, dtype=torch.bfloat16, device=cuda_dev)
    err = fai.error_word(cuda_dev.index)
    pkg.check_device_errors(cuda_dev.index)
    # this rank (0) is at epoch 5; rank 1 published 5: the GEMM runs
    signals = torch.tensor([5, 5, 5, 0, 0, 0, 0, 0], dtype=torch.int32, device=cuda_dev)
    assert _call(lib, a, w, out, signals, 2, 0, err, cuda_dev) == 0
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    _check(out, a, w)
    # rank 1 is still at epoch 4: its columns never become readable; the
    # wait runs out after its bound and the error word reports it
    signals = torch.tensor([5, 4, 5, 0, 0, 0, 0, 0], dtype=torch.int32, device=cuda_dev)
    t0 = time.perf_counter()
    assert _call(lib, a, w, out, signals, 2, 0, err, cuda_dev) == 0
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 >= 1.0
    assert int(err.item()) == 1  # LA_DEVERR_WAIT_TIMEOUT
    with pytest.raises(_lib.LeanAttnError, match="bounded wait timed out"):
        pkg.check_device_errors(cuda_dev.index)
    # the context is still usable
    signals[1] = 5
    assert _call(lib, a, w, out, signals, 2, 0, err, cuda_dev) == 0
    torch.cuda.synchronize()
    pkg.check_device_errors(cuda_dev.index)
    _check(out, a, w)


def test_o_proj_argument_errors(pkg, cuda_dev):
    from lean_infer_b200 import _lib

    lib = _lib.load()
    a = torch.zeros(4, 2048, dtype=torch.bfloat16, device=cuda_dev)
    w = torch.zeros(1024, 2048, dtype=torch.bfloat16, device=cuda_dev)
    out = torch.zeros(4, 1024, dtype=torch.bfloat16, device=cuda_dev)
    sig = torch.zeros(8, dtype=torch.int32, device=cuda_dev)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    s = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    # k not a multiple of 64 * world (2048 over 3 ranks), n not a multiple of 32
    assert lib.la_o_proj_gathered(p(a), 2048, p(w), 2048, p(out), 1024, 4, 1024, 2048, p(sig), 3, 0, p(err), s) == 2
    assert lib.la_o_proj_gathered(p(a), 2048, p(w), 2048, p(out), 1024, 4, 1000, 2048, p(sig), 1, 0, p(err), s) == 2
    # rank outside the world, null signals
    assert lib.la_o_proj_gathered(p(a), 2048, p(w), 2048, p(out), 1024, 4, 1024, 2048, p(sig), 2, 2, p(err), s) == 1
    assert lib.la_o_proj_gathered(p(a), 2048, p(w), 2048, p(out), 1024, 4, 1024, 2048, None, 1, 0, p(err), s) == 1
    # misaligned rows
    assert lib.la_o_proj_gathered(p(a), 2047, p(w), 2048, p(out), 1024, 4, 1024, 2048, p(sig), 1, 0, p(err), s) == 3
