"""la_paged_decode_noalloc, the decode entry point that allocates nothing,
against la_paged_decode, both called through the C ABI.

Some callers cannot allocate device memory where they run decode attention:
a host framework that owns every device allocation, a runtime that only
hands out a fixed arena, or a latency-bound loop where an allocation would
synchronise the device. The allocation-free
entry point keeps the split-KV partials in a fixed array inside the library
instead of a caller workspace; its results must match the workspace form's.

This file is collected last, so a failure here stops a `-x` run only after
every other test has run. It passes alone in a fresh process as well."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-2  # the decode tests' bound on bf16 outputs


def _args(w, out, lse):
    q, kc = w.q, w.k_cache
    return [
        ctypes.c_void_p(q.data_ptr()), q.stride(0), q.stride(2),
        ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(w.v_cache.data_ptr()),
        kc.stride(0), kc.stride(1), kc.stride(2), kc.shape[0], kc.shape[1],
        ctypes.c_void_p(w.block_table.data_ptr()), w.block_table.stride(0), w.block_table.shape[1],
        ctypes.c_void_p(w.cache_seqlens.data_ptr()),
        q.shape[0], q.shape[2], kc.shape[2], q.shape[3],
        ctypes.c_float(q.shape[3] ** -0.5),
        ctypes.c_void_p(out.data_ptr()), out.stride(0), out.stride(2),
        ctypes.c_void_p(lse.data_ptr()),
    ]


def test_noalloc_matches_workspace_entry_point(pkg, cuda_dev):
    from lean_infer_b200 import _lib
    from lean_infer_b200 import workloads as W

    lib = _lib.load()
    dev = cuda_dev.index
    assert lib.la_init(dev) == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    nbytes = ctypes.c_size_t(0)
    assert lib.la_paged_decode_workspace_size(dev, 16, 8, 128, ctypes.byref(nbytes)) == 0
    workspace = torch.empty(nbytes.value, dtype=torch.uint8, device=cuda_dev)

    # two calls in a row on different batches: sequences split across CTAs,
    # sequences finished inside one CTA, and a short batch after a long one
    batches = [W.decode_batch(128, 1, 1024, num_blocks=None, seed=51, device=cuda_dev),
               W.decode_batch(7, 300, 9000, num_blocks=None, seed=52, device=cuda_dev)]
    for w in batches:
        B, Hq = w.q.shape[0], w.q.shape[2]
        out_ref = torch.empty_like(w.q)
        lse_ref = torch.empty(B, Hq, dtype=torch.float32, device=cuda_dev)
        rc = lib.la_paged_decode(*_args(w, out_ref, lse_ref), ctypes.c_void_p(workspace.data_ptr()),
                                 ctypes.c_size_t(workspace.numel()), ctypes.c_void_p(err.data_ptr()), stream)
        assert rc == 0, _lib.status_string(rc)
        out = torch.full_like(w.q, float("nan"))
        lse = torch.full((B, Hq), float("nan"), dtype=torch.float32, device=cuda_dev)
        rc = lib.la_paged_decode_noalloc(*_args(w, out, lse), ctypes.c_void_p(err.data_ptr()), stream)
        assert rc == 0, _lib.status_string(rc)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.isfinite(out).all() and torch.isfinite(lse).all()
        assert (out.float() - out_ref.float()).abs().max().item() <= TOL
        assert (lse - lse_ref).abs().max().item() <= 1e-2
        # both entry points run the same kernels over the same split of the
        # keys, so the results are bit-identical, not only within tolerance
        assert torch.equal(out, out_ref) and torch.equal(lse, lse_ref)


def test_noalloc_rejects_beyond_its_array(pkg, cuda_dev):
    """A head count whose partials do not fit the fixed array is refused with
    LA_ERR_WORKSPACE (4) before anything is launched."""
    from lean_infer_b200 import _lib

    lib = _lib.load()
    null = ctypes.c_void_p(0)
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=cuda_dev)
    p = ctypes.c_void_p(dummy.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    # 64 query heads over 8 kv heads: 2 * #SMs * 64 * 129 * 4 bytes > 4 MiB
    rc = lib.la_paged_decode_noalloc(p, 64 * 128, 128, p, p, 256 * 8 * 128, 8 * 128, 128, 1, 256, p, 1, 1, p,
                                     1, 64, 8, 128, ctypes.c_float(0.088), p, 64 * 128, 128, null, null, stream)
    assert rc == 4
