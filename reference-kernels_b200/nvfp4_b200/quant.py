"""NVFP4 producer ops on the GPU: quantise fp16 / bf16 tensors into the
reference's input format, and convert block scales between the plain and the
128x4-blocked layouts (the ``to_blocked`` of
problems/nvidia/nvfp4_gemm/reference.py:12-24).

The outputs use the reference's ``input_t`` layouts, so a quantised operand
can be passed straight to ``custom_kernel``: packed values as a
``[rows, K/2, L]`` float4_e2m1fn_x2 view of contiguous ``(L, rows, K/2)``
storage, scales as the ``(32, 4, rows/128, 4, K/64, L)`` float8_e4m3fn
"permuted" view of the blocked storage (and, from ``to_plain``, a
``[rows, K/16, L]`` view of plain storage).
"""
from __future__ import annotations

import torch

from . import _lib
from .inputs import FP4X2, E4M3, permuted_view

_DTYPES = {torch.float16: 0, torch.bfloat16: 1}


def _stream(t):
    return torch._C._cuda_getCurrentRawStream(t.get_device())


def quantize(x: torch.Tensor, global_scale: float = 1.0):
    """x: [rows, K] or [rows, K, L] fp16/bf16 CUDA tensor with unit K stride
    (the [rows, K, L] form must be a view of contiguous (L, rows, K) storage).

    Returns (packed, scales): packed [rows, K/2, L] float4_e2m1fn_x2 and the
    blocked scales as the reference's permuted view.  Per 16-element block
    s = e4m3(amax / (6 g)), q = e2m1(x / (s g)) with round-to-nearest-even and
    saturation, g = global_scale, so that x ~= q * s * g."""
    if x.dim() == 2:
        x = x.unsqueeze(2)
    rows, k, l = x.shape
    if x.dtype not in _DTYPES or not x.is_cuda:
        raise _lib.Nvfp4Error("quantize: x must be an fp16 or bf16 CUDA tensor")
    if x.stride(1) != 1 or x.stride(0) != k:
        raise _lib.Nvfp4Error(f"quantize: x must have unit K stride and row stride K (strides {x.stride()})")
    packed = torch.empty((l, rows, k // 2), dtype=torch.uint8, device=x.device)
    blocked = torch.empty((l, rows // 128, k // 64, 32, 4, 4), dtype=torch.uint8, device=x.device)
    _lib.check(_lib.load().nvfp4_quantize(
        x.data_ptr(), _DTYPES[x.dtype], packed.data_ptr(), blocked.data_ptr(), rows, k, l, x.stride(2),
        rows * k // 2, rows * k // 16, float(global_scale), _stream(x)))
    return packed.permute(1, 2, 0).view(FP4X2), permuted_view(blocked.view(E4M3))


def to_blocked(plain: torch.Tensor) -> torch.Tensor:
    """Plain scales [rows, K/16, L] (or [rows, K/16]) -> the permuted view of blocked storage."""
    if plain.dim() == 2:
        plain = plain.unsqueeze(2)
    rows, sk, l = plain.shape
    if not plain.is_cuda or plain.element_size() != 1 or plain.stride(1) != 1:
        raise _lib.Nvfp4Error("to_blocked: plain scales must be a 1-byte CUDA tensor with unit column stride")
    out = torch.empty((l, rows // 128, sk // 4, 32, 4, 4), dtype=torch.uint8, device=plain.device)
    _lib.check(_lib.load().nvfp4_scales_to_blocked(
        plain.data_ptr(), out.data_ptr(), rows, sk, l, plain.stride(0), plain.stride(2), rows * sk, _stream(plain)))
    return permuted_view(out.view(E4M3))


def to_plain(permuted: torch.Tensor) -> torch.Tensor:
    """The reference's permuted (blocked) view -> plain scales [rows, K/16, L]."""
    rows = permuted.shape[2] * 128
    sk = permuted.shape[4] * 4
    l = permuted.shape[5]
    if permuted.stride()[:5] != (16, 4, (sk // 4) * 512, 1, 512):
        raise _lib.Nvfp4Error("to_plain: expected the permuted view of contiguous blocked storage")
    out = torch.empty((l, rows, sk), dtype=torch.uint8, device=permuted.device)
    _lib.check(_lib.load().nvfp4_scales_from_blocked(
        permuted.data_ptr(), out.data_ptr(), rows, sk, l, sk, rows * sk, permuted.stride(5), _stream(permuted)))
    return out.permute(1, 2, 0).view(E4M3)
