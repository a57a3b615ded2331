"""The TVM-FFI module of the library (libarcb200_tvm_ffi.so).

The reference's Python layer loads its GEMM as a TVM-FFI module and calls the typed
function with torch tensors (arc/mm.py:66-79: `_load_matmul()(a, b, out)`). This loads
the same kind of module for this library; its functions take torch (or any DLPack)
tensors:

    mod = arc.tvm_module.load()
    mod.matmul(a, b, out)                      # bf16 [M,K] x [N,K]^T -> [M,N]
    mod.a8w4_matmul(x, sa, wp, sb, out)        # int8 x packed int4, group-128 scales
    mod.fp8_fp4_gemm_nt(x, sfa, wp, sfw, out)  # e4m3 x e2m1, UE8M0 block scales

Each launches on the TVM-FFI environment stream of the output's device and raises on a
bad argument or a failed call. Building the module needs the tvm_ffi package
(`arc.build.build_tvm_ffi()`); nothing else in the package depends on it.
"""
from __future__ import annotations

import threading

from .build import TVM_FFI_LIB_PATH

_mod = None
_lock = threading.Lock()


def load():
    """The loaded module (loaded once per process)."""
    global _mod
    if _mod is None:
        with _lock:
            if _mod is None:
                import tvm_ffi

                if not TVM_FFI_LIB_PATH.exists():
                    raise RuntimeError(f"{TVM_FFI_LIB_PATH} is not built; build it with "
                                       "arc.build.build_tvm_ffi() (needs the tvm_ffi package)")
                _mod = tvm_ffi.load_module(str(TVM_FFI_LIB_PATH))
    return _mod


__all__ = ["load"]
