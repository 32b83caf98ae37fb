"""Loader for libnvfp4_b200.so (the C ABI declared in include/nvfp4_b200.h).

The shared library is built in-tree by ``build.py`` / ``csrc/Makefile``.  There
is no CPU fallback: if the library or a CUDA device is missing, every call
raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# NVFP4_B200_LIBRARY points at another build of the same C ABI (e.g. a variant
# built for an A/B timing on one GPU); the default is the in-tree library.
LIB_PATH = os.environ.get("NVFP4_B200_LIBRARY") or os.path.join(_HERE, "libnvfp4_b200.so")

EXPORTS = (
    "nvfp4_last_error",
    "nvfp4_abi_version",
    "nvfp4_device_status",
    "nvfp4_gemv",
    "nvfp4_gemm",
    "nvfp4_dual_gemm",
    "nvfp4_gemv_noalloc",
    "nvfp4_quantize",
    "nvfp4_scales_to_blocked",
    "nvfp4_scales_from_blocked",
    "nvfp4_gemv_call",
    "nvfp4_gemm_call",
    "nvfp4_dual_gemm_call",
)

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64

_lib = None


class GemvArgs(ctypes.Structure):
    """nvfp4_gemv_args of include/nvfp4_b200.h."""
    _fields_ = [("a", _P), ("b", _P), ("sfa_blk", _P), ("sfb_blk", _P), ("c", _P),
                ("M", ctypes.c_int32), ("K", ctypes.c_int32), ("L", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("a_lstride", _L), ("b_lstride", _L), ("sfa_lstride", _L), ("sfb_lstride", _L), ("c_lstride", _L),
                ("stream", _P)]


class GemmArgs(ctypes.Structure):
    """nvfp4_gemm_args of include/nvfp4_b200.h (b2 / sfb2_blk used by the dual GEMM only)."""
    _fields_ = [("a", _P), ("b", _P), ("b2", _P), ("sfa_blk", _P), ("sfb_blk", _P), ("sfb2_blk", _P), ("c", _P),
                ("M", ctypes.c_int32), ("N", ctypes.c_int32), ("K", ctypes.c_int32), ("L", ctypes.c_int32),
                ("a_lstride", _L), ("b_lstride", _L), ("sfa_lstride", _L), ("sfb_lstride", _L), ("ldc", _L),
                ("c_lstride", _L), ("stream", _P)]


class Nvfp4Error(RuntimeError):
    """Raised when an entry point of libnvfp4_b200.so returns a non-zero code."""


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise Nvfp4Error(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(nvcc, sm_100a); there is no CPU fallback")
    lib = ctypes.CDLL(LIB_PATH)
    lib.nvfp4_last_error.restype = ctypes.c_char_p
    lib.nvfp4_last_error.argtypes = []
    lib.nvfp4_abi_version.restype = _I
    lib.nvfp4_device_status.restype = _I
    lib.nvfp4_device_status.argtypes = [_I]
    lib.nvfp4_gemv.restype = _I
    lib.nvfp4_gemv.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _L, _L, _L, _L, _L, _P]
    lib.nvfp4_gemv_noalloc.restype = _I
    lib.nvfp4_gemv_noalloc.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _L, _L, _L, _L, _L, _P]
    lib.nvfp4_quantize.restype = _I
    lib.nvfp4_quantize.argtypes = [_P, _I, _P, _P, _I, _I, _I, _L, _L, _L, ctypes.c_float, _P]
    for name in ("nvfp4_scales_to_blocked", "nvfp4_scales_from_blocked"):
        getattr(lib, name).restype = _I
        getattr(lib, name).argtypes = [_P, _P, _I, _I, _I, _L, _L, _L, _P]
    lib.nvfp4_gemm.restype = _I
    lib.nvfp4_gemm.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _L, _L, _L, _L, _L, _L, _P]
    lib.nvfp4_dual_gemm.restype = _I
    lib.nvfp4_dual_gemm.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _L, _L, _L, _L, _L, _L, _P]
    lib.nvfp4_gemv_call.restype = _I
    lib.nvfp4_gemv_call.argtypes = [ctypes.POINTER(GemvArgs)]
    for name in ("nvfp4_gemm_call", "nvfp4_dual_gemm_call"):
        getattr(lib, name).restype = _I
        getattr(lib, name).argtypes = [ctypes.POINTER(GemmArgs)]
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != 0:
        msg = load().nvfp4_last_error().decode(errors="replace")
        raise Nvfp4Error(f"libnvfp4_b200 error {rc}: {msg}")


def device_status(clear: bool = True) -> int:
    """Device status word (bounded-wait timeouts in the GEMM kernels); 0 = ok."""
    return load().nvfp4_device_status(1 if clear else 0)
