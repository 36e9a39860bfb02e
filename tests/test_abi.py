"""The C-ABI library loads and exports every entry point the header declares
(no compute calls: this runs without a GPU)."""
import ctypes
import re

import pytest
import torch

from conftest import REPO

HEADER = REPO / "include" / "lean_attn.h"


def header_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(la_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(pkg):
    from lean_infer_b200 import _lib

    lib = _lib.load()
    syms = header_symbols()
    assert "la_paged_decode" in syms and "la_qk_norm_rope_paged_write" in syms
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, f"symbols declared in lean_attn.h but not exported: {missing}"
    # every declared entry point has a ctypes signature in the binding
    untyped = [s for s in syms if s not in _lib.exported_symbols() and s != "la_status_string"]
    assert not untyped, untyped


def test_version_and_status_strings(pkg):
    from lean_infer_b200 import _lib

    lib = _lib.load()
    m = re.search(r"#define LA_VERSION (\d+)", HEADER.read_text())
    assert lib.la_version() == int(m.group(1))
    assert _lib.status_string(0) == "ok"
    assert "workspace" in _lib.status_string(4)


def test_library_has_no_torch_dependency(pkg):
    """The .so is plain CUDA C++: it must not need libtorch to load."""
    from lean_infer_b200 import _lib

    data = _lib.LIB_PATH.read_bytes()
    assert b"libtorch" not in data and b"libc10" not in data


def test_cpu_tensors_are_rejected(pkg):
    q = torch.zeros(1, 1, 16, 128, dtype=torch.bfloat16)
    kc = torch.zeros(2, 256, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.flash_attn_with_kvcache(q, kc, kc, cache_seqlens=torch.ones(1, dtype=torch.int32),
                                    block_table=torch.zeros(1, 1, dtype=torch.int32))


def test_unsupported_arguments_raise(pkg):
    q = torch.zeros(1, 1, 16, 128, dtype=torch.bfloat16)
    kc = torch.zeros(2, 256, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        pkg.flash_attn_with_kvcache(q, kc, kc, k=q, v=q)
    with pytest.raises(NotImplementedError):
        pkg.flash_attn_with_kvcache(q, kc, kc, window_size=(8, 0))
    with pytest.raises(RuntimeError):  # q_len > 1 is chunked prefill: supported, but only on CUDA tensors
        pkg.flash_attn_with_kvcache(torch.zeros(1, 2, 16, 128, dtype=torch.bfloat16), kc, kc)


def test_argument_errors_before_launch(pkg):
    """Invalid arguments come back as status codes without touching a GPU."""
    from lean_infer_b200 import _lib

    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.la_paged_decode_workspace_size(0, 16, 3, 128, ctypes.byref(n)) == 1  # Hkv must divide 8
    assert lib.la_paged_decode_workspace_size(0, 16, 8, 64, ctypes.byref(n)) == 1   # head_dim 128 only
    null = ctypes.c_void_p(0)
    rc = lib.la_paged_decode(null, 0, 0, null, null, 0, 0, 0, 1, 256, null, 0, 1, null, 1, 16, 8, 128,
                             ctypes.c_float(0.1), null, 0, 0, null, null, 0, null, null)
    assert rc == 1
    # chunked prefill over the paged cache: null pointers, a block size that
    # 64-key tiles cannot walk, and an inconsistent uniform q_len
    fake = ctypes.c_void_p(1 << 20)

    def paged(q=fake, bs=256, q_len=4, T=8):
        return lib.la_prefill_paged(q, 2048, 128, fake, fake, 256 * 1024, 1024, 128, 4, bs, fake, 2, 2, fake, null,
                                    q_len, 2, 4, T, 16, 8, 128, ctypes.c_float(0.1), 1, fake, 2048, 128, null, null,
                                    null)

    assert paged(q=null) == 1
    assert paged(bs=48) == 2
    assert paged(T=9) == 1
    assert paged(q_len=0, T=0) == 0  # nothing to do


def test_glue_argument_checks(pkg):
    """The fused glue kernels validate before launching (no GPU needed)."""
    from lean_infer_b200 import _lib

    lib = _lib.load()
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(1 << 20)
    # a null addend is allowed: only the given pointers' strides are checked
    assert lib.la_add_rms_norm(fake, 1024, null, 0, null, 0, fake, 1024, fake, 0, 1024, ctypes.c_float(1e-6), null) == 0
    assert lib.la_add_rms_norm(null, 1024, null, 0, null, 0, fake, 1024, fake, 4, 1024, ctypes.c_float(1e-6), null) == 1
    assert lib.la_add_rms_norm(fake, 1024, null, 0, null, 0, fake, 1024, fake, 4, 1020, ctypes.c_float(1e-6), null) == 2
    assert lib.la_add_rms_norm(fake, 1000, null, 0, null, 0, fake, 1024, fake, 4, 1024, ctypes.c_float(1e-6), null) == 3
    assert lib.la_silu_mul(fake, 6144, fake, 3072, 0, 3072, null) == 0
    assert lib.la_silu_mul(fake, 6000, fake, 3072, 4, 3072, null) == 3
    # argmax rows: no rows is a no-op; empty rows, short strides, null or
    # misaligned pointers are rejected before any launch
    assert lib.la_argmax_rows(fake, 151936, 0, 151936, fake, null) == 0
    assert lib.la_argmax_rows(null, 151936, 4, 151936, fake, null) == 1
    assert lib.la_argmax_rows(fake, 151936, 4, 0, fake, null) == 1
    assert lib.la_argmax_rows(fake, 100, 4, 151936, fake, null) == 1
    assert lib.la_argmax_rows(ctypes.c_void_p((1 << 20) + 1), 151936, 4, 151936, fake, null) == 3
    assert lib.la_argmax_rows(fake, 151936, 4, 151936, ctypes.c_void_p((1 << 20) + 4), null) == 3
