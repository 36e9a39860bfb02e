"""ctypes binding of liblean_attn.so (declared in include/lean_attn.h).

Loading fails loudly: there is no CPU or torch fallback for any kernel. Every
wrapped call raises ``LeanAttnError`` (a RuntimeError) when the library
returns a non-zero la_status.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblean_attn.so"

LA_OK = 0
DEVERR_NAMES = {
    0: "ok",
    1: "bounded wait timed out",
    2: "block id outside the pool",
    3: "sequence longer than its block table",
    4: "position outside the rope table",
    5: "shared memory base misaligned",
}


class LeanAttnError(RuntimeError):
    pass


_c_int_p = POINTER(c_int)

# name -> argtypes (restype is int for all)
_SIGNATURES = {
    "la_version": [],
    "la_last_cuda_error": [],
    "la_init": [c_int],
    "la_qk_norm_rope_paged_write": [
        c_void_p, c_int64, c_int64,
        c_void_p, c_int64, c_int64,
        c_void_p, c_int64, c_int64,
        c_void_p, c_void_p, c_float,
        c_void_p, c_void_p, c_int64,
        c_void_p, c_void_p,
        c_int, c_int, c_int64,
        c_void_p, c_int64, c_int,
        c_void_p, c_void_p,
        c_int64, c_int64, c_int64,
        c_int64, c_int,
        c_void_p, c_int64, c_int64,
        c_void_p, c_int64, c_int64,
        c_int, c_int, c_int,
        c_void_p, c_void_p,
    ],
    "la_paged_kv_write": [
        c_void_p, c_int64, c_int64,
        c_void_p, c_int64, c_int64,
        c_void_p, c_void_p,
        c_int, c_int, c_int64,
        c_void_p, c_int64, c_int,
        c_void_p, c_void_p,
        c_int64, c_int64, c_int64,
        c_int64, c_int,
        c_int, c_int,
        c_void_p, c_void_p,
    ],
    "la_paged_decode_workspace_size": [c_int, c_int, c_int, c_int, POINTER(c_size_t)],
    "la_paged_decode": [
        c_void_p, c_int64, c_int64,
        c_void_p, c_void_p,
        c_int64, c_int64, c_int64,
        c_int64, c_int,
        c_void_p, c_int64, c_int,
        c_void_p,
        c_int, c_int, c_int, c_int,
        c_float,
        c_void_p, c_int64, c_int64,
        c_void_p,
        c_void_p, c_size_t,
        c_void_p, c_void_p,
    ],
    "la_paged_decode_noalloc": [
        c_void_p, c_int64, c_int64,
        c_void_p, c_void_p,
        c_int64, c_int64, c_int64,
        c_int64, c_int,
        c_void_p, c_int64, c_int,
        c_void_p,
        c_int, c_int, c_int, c_int,
        c_float,
        c_void_p, c_int64, c_int64,
        c_void_p,
        c_void_p, c_void_p,
    ],
    "la_paged_decode_allgather": [
        c_void_p, c_int64, c_int64,
        c_void_p, c_void_p,
        c_int64, c_int64, c_int64,
        c_int64, c_int,
        c_void_p, c_int64, c_int,
        c_void_p,
        c_int, c_int, c_int, c_int,
        c_float,
        c_void_p, c_int64, c_int64,
        c_int, c_int,
        c_void_p, c_size_t,
        c_void_p, c_void_p,
    ],
    "la_p2p_barrier": [c_void_p, c_int, c_int, c_void_p, c_void_p],
    "la_p2p_publish": [c_void_p, c_int, c_int, c_void_p, c_void_p],
    "la_o_proj_gathered": [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int,
                           c_void_p, c_int, c_int, c_void_p, c_void_p],
    "la_p2p_alloc": [c_size_t, POINTER(c_void_p), c_void_p],
    "la_p2p_open": [c_void_p, POINTER(c_void_p)],
    "la_p2p_close": [c_void_p],
    "la_p2p_free": [c_void_p],
    "la_prefill_varlen": [
        c_void_p, c_int64, c_int64,
        c_void_p, c_int64, c_int64,
        c_void_p, c_int64, c_int64,
        c_void_p, c_int, c_int, c_int64,
        c_int, c_int, c_int,
        c_float, c_int,
        c_void_p, c_int64, c_int64,
        c_void_p,
        c_void_p, c_void_p,
    ],
    "la_add_rms_norm": [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
                        c_int64, c_int, c_float, c_void_p],
    "la_silu_mul": [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_void_p],
    "la_argmax_rows": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "la_prefill_paged": [
        c_void_p, c_int64, c_int64,
        c_void_p, c_void_p,
        c_int64, c_int64, c_int64,
        c_int64, c_int,
        c_void_p, c_int64, c_int,
        c_void_p,
        c_void_p, c_int, c_int, c_int, c_int64,
        c_int, c_int, c_int,
        c_float, c_int,
        c_void_p, c_int64, c_int64,
        c_void_p,
        c_void_p, c_void_p,
    ],
}

_lib = None


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load liblean_attn.so once; raise if it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise LeanAttnError(
            f"{LIB_PATH} is missing: build it first (python -c 'import __graft_entry__ as g; g.build()')"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, argtypes in _SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue  # checked by tests against the header
        fn.argtypes = argtypes
        fn.restype = c_int
    lib.la_status_string.argtypes = [c_int]
    lib.la_status_string.restype = ctypes.c_char_p
    _lib = lib
    return lib


def status_string(code: int) -> str:
    return load().la_status_string(code).decode()


def check(code: int, what: str) -> None:
    if code != LA_OK:
        lib = load()
        extra = ""
        if code == 5:  # LA_ERR_CUDA
            extra = f" (cudaError {lib.la_last_cuda_error()})"
        raise LeanAttnError(f"{what} failed: {status_string(code)}{extra}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
