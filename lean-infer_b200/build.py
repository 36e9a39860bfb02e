"""Builds liblean_attn.so (the C-ABI library of the sm_100a kernels) in-tree.

The library is plain CUDA C++ compiled by nvcc for sm_100a only; it does not
link against torch. It is written to ``<package>/_lib/liblean_attn.so`` so it
travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "liblean_attn.so"

SOURCES = ["la_host.cu", "la_pre_attn.cu", "la_decode.cu", "la_decode_noalloc.cu", "la_prefill.cu", "la_p2p.cu", "la_elementwise.cu", "la_oproj.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build liblean_attn.so")
    return cand


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    return files


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel source into liblean_attn.so (sm_100a, -lineinfo)."""
    if not force and not needs_build():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = [str(CSRC / s) for s in SOURCES if (CSRC / s).exists()]
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), "-O3", "-std=c++17", *ARCH_FLAGS, "-lineinfo",
        "-Xcompiler", "-fPIC", "-shared", "-I", str(INCLUDE), "-I", str(CSRC),
        "-o", str(tmp), *srcs,
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}")
    if verbose:
        print(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
