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
PROBE_LIB_PATH = PKG_DIR / "libarcb200_probe.so"
TVM_FFI_LIB_PATH = PKG_DIR / "libarcb200_tvm_ffi.so"
TVM_FFI_SOURCE = "tvm_ffi_shim.cc"
STAMP = ROOT / "_build" / "libarcb200.hash"

SOURCES = ["api.cu"]
HEADERS = ["sm100.cuh", "peer_barrier.cuh", "gemm_bf16.cuh", "gemm_bf16_pair.cuh", "gemm_a8w4.cuh", "gemm_a8w4_decode.cuh", "quantize.cuh",
           "gemm_fp8fp4.cuh", "gemm_fp8fp4_pair.cuh", "prepack.cuh"]

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


def source_hash(probe: bool = False) -> str:
    h = hashlib.sha256(b"probe" if probe else b"")
    for name in SOURCES + HEADERS:
        h.update(name.encode())
        h.update((CSRC / name).read_bytes())
    h.update((INCLUDE / "arc_b200.h").read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def _paths(probe: bool):
    if probe:
        return PROBE_LIB_PATH, STAMP.with_name("libarcb200_probe.hash")
    return LIB_PATH, STAMP


def is_current(probe: bool = False) -> bool:
    lib, stamp = _paths(probe)
    return lib.exists() and stamp.exists() and stamp.read_text().strip() == source_hash(probe)


def build(force: bool = False, verbose: bool = False, probe: bool = False) -> Path:
    """Compile libarcb200.so in-tree (next to this file). Returns its path.

    probe=True builds libarcb200_probe.so with -DARC_PROBE (pipeline timestamps).
    """
    lib, stamp = _paths(probe)
    if not force and is_current(probe):
        return lib
    nvcc = find_nvcc()
    stamp.parent.mkdir(parents=True, exist_ok=True)
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc, *NVCC_FLAGS, *(["-DARC_PROBE"] if probe else []), "-I", str(INCLUDE),
           "-I", str(CSRC), "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout + res.stderr)
    (ROOT / "_build" / ("ptxas_probe.log" if probe else "ptxas.log")).write_text(
        res.stdout + res.stderr)
    tmp.replace(lib)
    stamp.write_text(source_hash(probe))
    return lib


def build_tvm_ffi(force: bool = False) -> Path | None:
    """Compile libarcb200_tvm_ffi.so: TVM-FFI typed exports (matmul, a8w4_matmul,
    fp8_fp4_gemm_nt) over the C ABI, the binding shape of the reference
    (arc/mm.py:30,48). Host C++ only (g++), linked against libarcb200.so, libtvm_ffi.so
    and the CUDA runtime. Returns None when the tvm_ffi package is not installed: the
    C ABI and the ctypes layer do not depend on it.
    """
    try:
        import tvm_ffi.libinfo as info
    except ImportError:
        return None
    lib = build()
    src = CSRC / TVM_FFI_SOURCE
    stamp = STAMP.with_name("libarcb200_tvm_ffi.hash")
    h = hashlib.sha256(src.read_bytes() + (INCLUDE / "arc_b200.h").read_bytes()).hexdigest()
    if not force and TVM_FFI_LIB_PATH.exists() and stamp.exists() and stamp.read_text().strip() == h:
        return TVM_FFI_LIB_PATH
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler for the TVM-FFI shim")
    cuda_home = Path(find_nvcc()).resolve().parent.parent
    tvm_lib = Path(info.find_libtvm_ffi()).parent
    tmp = TVM_FFI_LIB_PATH.with_suffix(".so.tmp")
    cmd = [cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-o", str(tmp), str(src),
           "-I", str(INCLUDE), "-I", info.find_include_path(), "-I", info.find_dlpack_include_path(),
           "-I", str(cuda_home / "include"),
           "-L", str(lib.parent), "-larcb200", "-L", str(tvm_lib), "-ltvm_ffi",
           "-L", str(cuda_home / "lib64"), "-lcudart",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tvm_lib}", f"-Wl,-rpath,{cuda_home / 'lib64'}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"TVM-FFI shim build failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    tmp.replace(TVM_FFI_LIB_PATH)
    stamp.parent.mkdir(parents=True, exist_ok=True)
    stamp.write_text(h)
    return TVM_FFI_LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(force=True, verbose=True, probe="--probe" in sys.argv))
    print(build_tvm_ffi(force=True))
