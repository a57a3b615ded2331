"""ctypes binding of libarcb200.so (the C ABI declared in include/arc_b200.h).

There is no fallback: if the library is missing or fails to load, every GEMM call
raises. Building it is `python -m arc.build` (or `__graft_entry__.build()`).
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH, PROBE_LIB_PATH

ARC_OK = 0
ARC_ERR_INVALID_ARGUMENT = 1
ARC_ERR_UNSUPPORTED = 2
ARC_ERR_CUDA = 3
ARC_ERR_NO_DEVICE = 4
ARC_ERR_DEVICE_TIMEOUT = 5

# Bits of arc_device_status (arc-gemm_b200/csrc/sm100.cuh): which kind of wait timed out.
STATUS_TIMEOUT_PEER = 1 << 6


class ArcError(RuntimeError):
    """A nonzero arc_status_t from the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class Plan(ctypes.Structure):
    _fields_ = [
        ("split", ctypes.c_int),
        ("token_tile", ctypes.c_int),
        ("weight_rows", ctypes.c_int),
        ("k_split", ctypes.c_int),
        ("grid", ctypes.c_int),
        ("load_stages", ctypes.c_int),
        ("groups_per_stage", ctypes.c_int),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


# Every symbol include/arc_b200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
SIGNATURES = {
    "arc_version": ([], _I),
    "arc_status_string": ([_I], ctypes.c_char_p),
    "arc_last_error": ([], ctypes.c_char_p),
    "arc_matmul_bf16": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _P], _I),
    "arc_a8w4_gemm": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P], _I),
    "arc_a8w4_describe_plan": ([_I, _I, _I, _I, ctypes.POINTER(Plan)], _I),
    "arc_device_status": ([_I, ctypes.POINTER(ctypes.c_uint32), _I], _I),
    "arc_probe_attach": ([_P, ctypes.c_size_t], _I),
    "arc_quantize_int8": ([_P, _P, _P, _I, _I, _I, _I, _P], _I),
    "arc_fp8_fp4_gemm": ([_P, _P, _P, _P, _P, _I, _I, _I, _P], _I),
    "arc_kernel_name": ([_I, _I, _I, _I, ctypes.c_char_p, _I], _I),
    "arc_fp8_fp4_gemm_ws": ([_P, _P, _P, _P, _P, _I, _I, _I, _P, ctypes.c_size_t, _P], _I),
    "arc_fp8_fp4_workspace_bytes": ([_I, _I, _I, ctypes.POINTER(ctypes.c_size_t)], _I),
    "arc_fp8_fp4_gemm_noalloc": ([_P, _P, _P, _P, _P, _I, _I, _I, _P], _I),
    "arc_a8w4_gemm_gather": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "arc_peer_barrier": ([_P, _I, _I, _P], _I),
    "arc_peer_barrier_ex": ([_P, _I, _I, ctypes.c_uint64, _P], _I),
    "arc_ipc_export": ([_P, _P, ctypes.POINTER(ctypes.c_uint64)], _I),
    "arc_ipc_open": ([_P, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)], _I),
    "arc_ipc_close": ([_P], _I),
    "arc_a8w4_prepack_weights": ([_P, _P, _I, _I, _P], _I),
    "arc_a8w4_gemm_prepacked": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _P], _I),
    "arc_a8w4_gemm_ex": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_uint, _P, _P], _I),
    "arc_a8w4_gemm_gather_ex": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_uint, _P], _I),
    "arc_a8w4_gemm_gather_sync": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_uint, _P], _I),
}

# Flags of arc_a8w4_gemm_ex / arc_a8w4_gemm_gather_ex (include/arc_b200.h).
A8W4_PREPACKED = 1
A8W4_STATIC_WEIGHTS = 2

# Operation codes of arc_kernel_name (include/arc_b200.h).
OP_MATMUL_BF16, OP_A8W4, OP_FP8_FP4 = 0, 1, 2


def probe_enabled() -> bool:
    """ARC_PROBE in the environment selects the probe build (as the reference does)."""
    return "ARC_PROBE" in os.environ

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded native library (loaded once per process)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                path = PROBE_LIB_PATH if probe_enabled() else LIB_PATH
                if not path.exists():
                    raise RuntimeError(
                        f"{path} is not built; the arc GEMMs have no fallback. "
                        "Build it with `python -m arc.build` (`--probe` for the probe build).")
                handle = ctypes.CDLL(str(path))
                for name, (argtypes, restype) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = argtypes
                    fn.restype = restype
                _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != ARC_OK:
        L = lib()
        detail = L.arc_last_error().decode(errors="replace")
        kind = L.arc_status_string(status).decode(errors="replace")
        raise ArcError(status, f"{what}: {kind}: {detail}")


def describe_plan(M: int, N: int, K: int, num_sms: int = 148) -> dict:
    """The A8W4 work decomposition for a shape (host-only)."""
    plan = Plan()
    check(lib().arc_a8w4_describe_plan(M, N, K, num_sms, ctypes.byref(plan)),
          "arc_a8w4_describe_plan")
    return plan.as_dict()


def kernel_name(op: int, M: int, N: int, K: int) -> str:
    """Name of the kernel launched for an operation of this shape on the current device
    (op: OP_MATMUL_BF16, OP_A8W4 or OP_FP8_FP4), as ncu lists it."""
    buf = ctypes.create_string_buffer(128)
    check(lib().arc_kernel_name(op, M, N, K, buf, len(buf)), "arc_kernel_name")
    return buf.value.decode()


def device_status(device: int, clear: bool = True) -> int:
    """Bit mask of kernel waits that timed out on `device` (synchronises it)."""
    val = ctypes.c_uint32(0)
    check(lib().arc_device_status(device, ctypes.byref(val), 1 if clear else 0),
          "arc_device_status")
    return int(val.value)


def probe_attach(buffer) -> None:
    """Attach a device buffer (a torch int64 CUDA tensor, or None) for probe stamps."""
    if buffer is None:
        check(lib().arc_probe_attach(None, 0), "arc_probe_attach")
    else:
        check(lib().arc_probe_attach(buffer.data_ptr(), buffer.numel() * buffer.element_size()),
              "arc_probe_attach")


def version() -> int:
    return int(lib().arc_version())
