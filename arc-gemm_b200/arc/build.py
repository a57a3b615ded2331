"""Ahead-of-time build of libarcb200.so for sm_100a.

Replaces the reference's JIT layer (arc/jit.py:176-275, which hashes the kernel
headers, runs nvcc through tvm_ffi.cpp.load_inline on the first call and targets the
family arch `10.0f`, arc/jit.py:302-319). Here the whole library is one nvcc
invocation for the arch-specific target `sm_100a` (tcgen05.mma kind::i8 needs the
`a` target), done once at build time. A content hash of the sources and flags is kept
next to the build products so an unchanged tree is not rebuilt (the role of
arc/jit.py:121-138 `hash_files`).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB_PATH = PKG_DIR / "libarcb200.so"
STAMP = ROOT / "_build" / "libarcb200.hash"

SOURCES = ["api.cu"]
HEADERS = ["sm100.cuh", "gemm_bf16.cuh", "gemm_a8w4.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-shared",
    "-Xptxas", "-v",
]


def find_nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"),
                 os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or CUDA_HOME")


def source_hash() -> str:
    h = hashlib.sha256()
    for name in SOURCES + HEADERS:
        h.update(name.encode())
        h.update((CSRC / name).read_bytes())
    h.update((INCLUDE / "arc_b200.h").read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def is_current() -> bool:
    return LIB_PATH.exists() and STAMP.exists() and STAMP.read_text().strip() == source_hash()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile libarcb200.so in-tree (next to this file). Returns its path."""
    if not force and is_current():
        return LIB_PATH
    nvcc = find_nvcc()
    STAMP.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-o", str(tmp),
           *[str(CSRC / s) for s in SOURCES]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout + res.stderr)
    (ROOT / "_build" / "ptxas.log").write_text(res.stdout + res.stderr)
    tmp.replace(LIB_PATH)
    STAMP.write_text(source_hash())
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
