"""``custom_kernel`` drop-ins for the three NVFP4 problems.

Each function keeps the reference's plugin contract ``custom_kernel(data:
input_t) -> output_t`` (``problems/nvidia/<problem>/task.py``): it takes the
tuple produced by ``generate_input``, launches the sm_100a kernel on the
current CUDA stream, writes into the preallocated output ``c`` and returns it.
Tensors are read through their data pointers and strides; nothing is copied,
allocated or synchronised on the call path.

Reference entry points replaced:
  gemv       problems/nvidia/nvfp4_gemv/submission.py:28-54 (and template_cute.py:199-247)
  gemm       problems/nvidia/nvfp4_gemm/submission.py:708-761
  dual_gemm  problems/nvidia/nvfp4_dual_gemm/submission.py:894-957
"""
from __future__ import annotations

import ctypes
import os
import weakref

import torch

from . import _lib

_CHECK_STATUS = os.environ.get("NVFP4_CHECK_STATUS", "0") == "1"


_raw_stream = torch._C._cuda_getCurrentRawStream


def _stream_ptr(t: torch.Tensor) -> int:
    # torch.cuda.current_stream() builds a Python Stream object (~3 us); the
    # raw getter returns the same cudaStream_t handle.
    return _raw_stream(t.get_device())


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise _lib.Nvfp4Error(msg)


def _check_operand(t: torch.Tensor, name: str) -> None:
    # [rows, K/2, L] view of contiguous (L, rows, K/2) storage (task.py input_t)
    st = t.stride()
    if t.is_cuda and st[1] == 1 and st[0] == t.shape[1] and t.element_size() == 1:
        return
    _require(t.is_cuda, f"{name} must be a CUDA tensor (no CPU fallback)")
    _require(t.element_size() == 1, f"{name} must be packed fp4x2 / uint8")
    _require(False, f"{name} must have K-major rows (strides {st})")


def _blocked_lstride(t: torch.Tensor, rows: int, sk: int, name: str) -> int:
    """Batch stride (bytes) of a permuted / blocked scale view; validates its strides."""
    kk = sk // 4
    st = t.stride()
    if len(st) == 6 and st[:5] == (16, 4, kk * 512, 1, 512) and t.shape[2] * 128 == rows and t.shape[4] == kk \
            and t.element_size() == 1:
        return st[5]  # fast path: the reference's permuted view
    _require(t.is_cuda and t.element_size() == 1, f"{name} must be fp8-e4m3 / uint8 on CUDA")
    if t.dim() == 6:
        # (32, 4, rows/128, 4, SK/4, L) view of (L, rows/128, SK/4, 32, 4, 4) storage
        _require(tuple(t.shape[:5]) == (32, 4, rows // 128, 4, kk),
                 f"{name}: blocked scale shape {tuple(t.shape)} does not match rows={rows}, K/16={sk}")
        _require(t.stride()[:5] == (16, 4, kk * 512, 1, 512),
                 f"{name}: blocked scales must be the reference's permuted view (strides {t.stride()})")
        return t.stride(5)
    # flat blocked vector (to_blocked output) for L == 1
    _require(t.dim() == 1 and t.numel() == rows * sk and t.stride(0) == 1,
             f"{name}: expected a (32,4,*,4,*,L) permuted view or a flat to_blocked vector")
    return rows * sk


def _post():
    if _CHECK_STATUS:
        torch.cuda.synchronize()
        st = _lib.device_status(True)
        if st != 0:
            raise _lib.Nvfp4Error(f"kernel pipeline wait timed out (device status {st})")


def _gemv_args(data):
    a, b, _sfa, _sfb, sfa_p, sfb_p, c = data
    m, k2, l = a.shape
    k = 2 * k2
    _check_operand(a, "a")
    _require(b.is_cuda and b.stride(1) == 1 and b.shape[1] == k2 and b.shape[2] == l, "b must be [rows, K/2, L]")
    _require(c.dtype == torch.float16 and tuple(c.shape) == (m, 1, l), "c must be fp16 [M, 1, L]")
    sa = _blocked_lstride(sfa_p, m, k // 16, "sfa_permuted")
    sb = _blocked_lstride(sfb_p, sfb_p.shape[2] * 128 if sfb_p.dim() == 6 else 128, k // 16, "sfb_permuted")
    return _lib.load().nvfp4_gemv_call, _lib.GemvArgs(
        a.data_ptr(), b.data_ptr(), sfa_p.data_ptr(), sfb_p.data_ptr(), c.data_ptr(),
        m, k, l, 0, a.stride(2), b.stride(2), sa, sb, c.stride(2), None)


def _gemm_args(data):
    a, b, _sfa, _sfb, sfa_p, sfb_p, c = data
    m, k2, l = a.shape
    n = b.shape[0]
    k = 2 * k2
    _check_operand(a, "a")
    _check_operand(b, "b")
    _require(c.dtype == torch.float16 and tuple(c.shape) == (m, n, l) and c.stride(1) == 1,
             "c must be fp16 [M, N, L] with unit column stride")
    sa = _blocked_lstride(sfa_p, m, k // 16, "sfa_permuted")
    sb = _blocked_lstride(sfb_p, n, k // 16, "sfb_permuted")
    return _lib.load().nvfp4_gemm_call, _lib.GemmArgs(
        a.data_ptr(), b.data_ptr(), None, sfa_p.data_ptr(), sfb_p.data_ptr(), None, c.data_ptr(),
        m, n, k, l, a.stride(2), b.stride(2), sa, sb, c.stride(0), c.stride(2), None)


def _dual_args(data):
    a, b1, b2, _sfa, _sfb1, _sfb2, sfa_p, sfb1_p, sfb2_p, c = data
    m, k2, l = a.shape
    n = b1.shape[0]
    k = 2 * k2
    _check_operand(a, "a")
    _check_operand(b1, "b1")
    _check_operand(b2, "b2")
    _require(b1.stride(2) == b2.stride(2), "b1 and b2 must share their batch stride")
    _require(c.dtype == torch.float16 and tuple(c.shape) == (m, n, l) and c.stride(1) == 1,
             "c must be fp16 [M, N, L] with unit column stride")
    sa = _blocked_lstride(sfa_p, m, k // 16, "sfa_permuted")
    sb1 = _blocked_lstride(sfb1_p, n, k // 16, "sfb1_permuted")
    sb2 = _blocked_lstride(sfb2_p, n, k // 16, "sfb2_permuted")
    _require(sb1 == sb2, "sfb1 and sfb2 must share their batch stride")
    return _lib.load().nvfp4_dual_gemm_call, _lib.GemmArgs(
        a.data_ptr(), b1.data_ptr(), b2.data_ptr(), sfa_p.data_ptr(), sfb1_p.data_ptr(), sfb2_p.data_ptr(),
        c.data_ptr(), m, n, k, l, a.stride(2), b1.stride(2), sa, sb1, c.stride(0), c.stride(2), None)


# Validated launch arguments per input tuple.  The reference harness calls
# custom_kernel on the same tuple objects many times; re-validating strides,
# re-reading the data pointers and converting 16 scalar ctypes arguments costs
# several microseconds per call.  Each entry keeps the packed argument block
# of the C ABI's *_call entry points, so a repeated call only stores the
# current stream into it.  An entry is used only while every tensor of the
# tuple is the very object it was built from (weak references), so a recycled
# id() never hits; a tensor whose storage is swapped in place (Tensor.set_)
# would not be noticed.
_CACHE: dict = {}
_CACHE_MAX = 256


_current_device = torch._C._cuda_getDevice


def _same_device(data) -> None:
    """Every tensor on one device, and that device the current one: the
    library takes its workspace, status word and tensor-map context from the
    current device, and the stream from the tensors' device."""
    dev = data[0].get_device()
    for i, t in enumerate(data):
        if isinstance(t, torch.Tensor) and t.is_cuda and t.get_device() != dev:
            _require(False, f"tuple slot {i} is on cuda:{t.get_device()}, slot 0 on cuda:{dev}")
    _require(dev == _current_device(),
             f"the tensors are on cuda:{dev} but cuda:{_current_device()} is current; "
             f"call inside torch.cuda.device({dev})")


def _dispatch(data, build):
    ent = _CACHE.get(id(data))
    if ent is not None:
        refs, fn, block, ref, dev = ent
        if all(r() is t for r, t in zip(refs, data)) and dev == _current_device():
            block.stream = _raw_stream(dev)
            rc = fn(ref)
            if rc:
                _lib.check(rc)
            if _CHECK_STATUS:
                _post()
            return data[-1]
    fn, block = build(data)
    _same_device(data)
    dev = data[0].get_device()
    ref = ctypes.byref(block)
    block.stream = _raw_stream(dev)
    _lib.check(fn(ref))
    if len(_CACHE) >= _CACHE_MAX:
        _CACHE.pop(next(iter(_CACHE)))
    _CACHE[id(data)] = (tuple(weakref.ref(t) for t in data), fn, block, ref, dev)
    _post()
    return data[-1]


def gemv(data):
    """custom_kernel for nvfp4_gemv: reads a, b and the blocked (permuted) scales, writes c[:, 0, :]."""
    return _dispatch(data, _gemv_args)


def gemm(data):
    """custom_kernel for nvfp4_gemm: reads a, b and the blocked (permuted) scales, writes c."""
    return _dispatch(data, _gemm_args)


def dual_gemm(data):
    """custom_kernel for nvfp4_dual_gemm: c = fp16(silu(A.B1^T) * (A.B2^T))."""
    return _dispatch(data, _dual_args)
