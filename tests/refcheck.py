"""Test helpers: the reference's ref_kernel restated on torch._scaled_mm (the
library call the reference itself makes) and the oracle on numpy copies."""
from __future__ import annotations

import numpy as np
import torch

from nvfp4_b200.inputs import to_blocked
from oracle import oracle


def u8(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.uint8).cpu().numpy() if t.dtype != torch.uint8 else t.cpu().numpy()


def scaled_mm_ref(problem: str, data):
    """ref_kernel of problems/nvidia/nvfp4_{gemv,gemm,dual_gemm}/reference.py on the GPU."""
    if problem == "dual":
        a, b1, b2, sfa, sfb1, sfb2, _, _, _, c = data
        m, n, l = c.shape
        out = torch.empty((m, n, l), dtype=torch.float16, device=c.device)
        for i in range(l):
            sa = to_blocked(sfa[:, :, i].contiguous())
            r1 = torch._scaled_mm(a[:, :, i], b1[:, :, i].transpose(0, 1), sa,
                                  to_blocked(sfb1[:, :, i].contiguous()), bias=None, out_dtype=torch.float32)
            r2 = torch._scaled_mm(a[:, :, i], b2[:, :, i].transpose(0, 1), sa,
                                  to_blocked(sfb2[:, :, i].contiguous()), bias=None, out_dtype=torch.float32)
            out[:, :, i] = (torch.nn.functional.silu(r1) * r2).to(torch.float16)
        return out
    a, b, sfa, sfb, _, _, c = data
    m, n, l = c.shape
    out = torch.empty_like(c)
    for i in range(l):
        res = torch._scaled_mm(a[:, :, i], b[:, :, i].transpose(0, 1),
                               to_blocked(sfa[:, :, i].contiguous()), to_blocked(sfb[:, :, i].contiguous()),
                               bias=None, out_dtype=torch.float16)
        if problem == "gemv":
            out[:, 0, i] = res[:, 0]
        else:
            out[:, :, i] = res
    return out


def oracle_ref(problem: str, data) -> np.ndarray:
    """The CPU oracle on host copies of the plain-layout tensors: fp16 [M, N, L]."""
    if problem == "dual":
        a, b1, b2, sfa, sfb1, sfb2, _, _, _, c = data
        m, n, l = c.shape
        out = np.empty((m, n, l), np.float16)
        for i in range(l):
            out[:, :, i] = oracle.ref_dual(u8(a[:, :, i]), u8(b1[:, :, i]), u8(b2[:, :, i]),
                                           u8(sfa[:, :, i]), u8(sfb1[:, :, i]), u8(sfb2[:, :, i]))
        return out
    a, b, sfa, sfb, _, _, c = data
    m, n, l = c.shape
    out = np.empty((m, n, l), np.float16)
    for i in range(l):
        if problem == "gemv":
            out[:, 0, i] = oracle.ref_gemv(u8(a[:, :, i]), u8(b[:, :, i]), u8(sfa[:, :, i]), u8(sfb[:, :, i]))
        else:
            out[:, :, i] = oracle.ref_gemm(u8(a[:, :, i]), u8(b[:, :, i]), u8(sfa[:, :, i]), u8(sfb[:, :, i]))
    return out


def assert_match(received, expected, what="", rtol=1e-3, atol=1e-3):
    """The reference tolerance (utils.py verbose_allclose, rtol=atol=1e-3)."""
    r = received.float().cpu().numpy() if isinstance(received, torch.Tensor) else received
    e = expected.float().cpu().numpy() if isinstance(expected, torch.Tensor) else expected
    rep = oracle.allclose_report(r, e, rtol=rtol, atol=atol)
    assert not rep, f"{what}: " + " | ".join(rep)
