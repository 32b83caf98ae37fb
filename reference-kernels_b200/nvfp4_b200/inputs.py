"""Seeded input tuples for the three NVFP4 problems.

Two generators:

* ``reference_input(problem, ...)`` restates ``generate_input`` of
  ``problems/nvidia/nvfp4_gemv/reference.py:57-166``,
  ``problems/nvidia/nvfp4_gemm/reference.py:56-158`` and
  ``problems/nvidia/nvfp4_dual_gemm/reference.py:80-196``: the same torch RNG
  calls in the same order and the same value distributions, so that on a CUDA
  device with the same seed it yields the reference's tensors bit for bit.  The
  permuted ("blocked") scale copies are built with a reshape instead of the
  reference's advanced-index scatter; the resulting memory order is the same.
* ``baseline_input(problem, ...)`` draws the distributions of the build's
  benchmark configurations: every packed byte uniform over 0..255 and every
  block scale uniform in [0.25, 2.0] rounded to e4m3fn.

Both return the reference's ``input_t`` tuple layout (``task.py`` of each
problem): tensors are views of contiguous ``(L, rows, cols)`` buffers permuted
to ``(rows, cols, L)``.
"""
from __future__ import annotations

import torch

SF_VEC = 16
FP4X2 = torch.float4_e2m1fn_x2
E4M3 = torch.float8_e4m3fn


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def blocked_from_plain(plain_lmk: torch.Tensor) -> torch.Tensor:
    """Plain scales stored (L, rows, SK) -> blocked storage (L, rows/128, SK/4, 32, 4, 4).

    The returned tensor is contiguous; its memory order per batch index equals
    ``to_blocked`` of ``nvfp4_gemm/reference.py:12-24``.
    """
    l, rows, sk = plain_lmk.shape
    assert rows % 128 == 0 and sk % 4 == 0, (rows, sk)
    v = plain_lmk.reshape(l, rows // 128, 4, 32, sk // 4, 4)  # (l, mm, mm4, mm32, kk, kk4)
    return v.permute(0, 1, 4, 3, 2, 5).contiguous()            # (l, mm, kk, mm32, mm4, kk4)


def permuted_view(blocked_storage: torch.Tensor) -> torch.Tensor:
    """(l, mm, kk, 32, 4, 4) storage -> the reference's (32, 4, mm, 4, kk, l) view."""
    return blocked_storage.permute(3, 4, 1, 5, 2, 0)


def to_blocked(plain_2d: torch.Tensor) -> torch.Tensor:
    """Torch restatement of ``to_blocked`` (reference.py:12-24): [rows, SK] -> flat."""
    return blocked_from_plain(plain_2d.unsqueeze(0)).reshape(-1)


def _scales_reference_like(l, mn, sf_k, device, kind):
    """create_scale_factor_tensors of the reference (same RNG consumption)."""
    shape = (l, mn, sf_k)
    if kind == "randint3":
        plain = torch.randint(0, 3, shape, dtype=torch.int8, device=device).to(E4M3)
    elif kind == "randint4":
        plain = torch.randint(0, 4, shape, dtype=torch.int8, device=device).to(E4M3)
    else:  # "rand": fp32 in [0, 1) cast to e4m3
        plain = torch.rand(shape, dtype=torch.float32, device=device).to(E4M3)
    mma_shape = (l, ceil_div(mn, 128), ceil_div(sf_k, 4), 32, 4, 4)
    # The reference draws (and then overwrites) a second tensor of this shape;
    # draw it too so the RNG stream stays aligned with the reference.
    if kind == "randint3":
        torch.randint(0, 3, mma_shape, dtype=torch.int8, device=device)
    elif kind == "randint4":
        torch.randint(0, 4, mma_shape, dtype=torch.int8, device=device)
    blocked = blocked_from_plain(plain.view(torch.uint8)).view(E4M3)
    return plain.permute(1, 2, 0), permuted_view(blocked)


def reference_input(problem: str, m: int, k: int, l: int, seed: int, n: int | None = None,
                    device="cuda"):
    torch.manual_seed(seed)
    sf_k = ceil_div(k, SF_VEC)
    if problem == "gemv":
        a = torch.randint(0, 4, (l, m, k // 2), dtype=torch.uint8, device=device).permute(1, 2, 0)
        b = torch.randint(0, 4, (l, 128, k // 2), dtype=torch.uint8, device=device).permute(1, 2, 0)
        c = torch.randn((l, m, 1), dtype=torch.float16, device=device).permute(1, 2, 0)
        sfa, sfa_p = _scales_reference_like(l, m, sf_k, device, "randint3")
        sfb, sfb_p = _scales_reference_like(l, 128, sf_k, device, "randint3")
        return (a.view(FP4X2), b.view(FP4X2), sfa, sfb, sfa_p, sfb_p, c)
    if problem == "gemm":
        a = torch.randint(-128, 128, (l, m, k // 2), dtype=torch.int8, device=device).permute(1, 2, 0)
        b = torch.randint(-128, 128, (l, n, k // 2), dtype=torch.int8, device=device).permute(1, 2, 0)
        c = torch.randn((l, m, n), dtype=torch.float16, device=device).permute(1, 2, 0)
        sfa, sfa_p = _scales_reference_like(l, m, sf_k, device, "randint4")
        sfb, sfb_p = _scales_reference_like(l, n, sf_k, device, "randint4")
        return (a.view(FP4X2), b.view(FP4X2), sfa, sfb, sfa_p, sfb_p, c)
    if problem == "dual":
        def fp4(mn):
            t = torch.randint(255, size=(l, mn, k // 2), dtype=torch.uint8, device=device)
            return (t & 0b1011_1011).permute(1, 2, 0).view(FP4X2)
        a, b1, b2 = fp4(m), fp4(n), fp4(n)
        c = torch.randn((l, m, n), dtype=torch.float16, device=device).permute(1, 2, 0)
        sfa, sfa_p = _scales_reference_like(l, m, sf_k, device, "rand")
        sfb1, sfb1_p = _scales_reference_like(l, n, sf_k, device, "rand")
        sfb2, sfb2_p = _scales_reference_like(l, n, sf_k, device, "rand")
        return (a, b1, b2, sfa, sfb1, sfb2, sfa_p, sfb1_p, sfb2_p, c)
    raise ValueError(problem)


def _uniform_bytes(gen, shape, device):
    return torch.randint(0, 256, shape, dtype=torch.uint8, device=device, generator=gen)


def _uniform_scales(gen, l, mn, sf_k, device):
    f = torch.empty((l, mn, sf_k), dtype=torch.float32, device=device).uniform_(0.25, 2.0, generator=gen)
    plain = f.to(E4M3)
    blocked = blocked_from_plain(plain.view(torch.uint8)).view(E4M3)
    return plain.permute(1, 2, 0), permuted_view(blocked)


def baseline_input(problem: str, m: int, k: int, l: int = 1, seed: int = 1111,
                   n: int | None = None, device="cuda"):
    """Uniform-byte / uniform-scale inputs (the build's benchmark distributions)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    sf_k = ceil_div(k, SF_VEC)
    if problem == "gemv":
        a = _uniform_bytes(gen, (l, m, k // 2), device).permute(1, 2, 0)
        b = torch.zeros((l, 128, k // 2), dtype=torch.uint8, device=device)
        b[:, 0] = _uniform_bytes(gen, (l, k // 2), device)
        c = torch.zeros((l, m, 1), dtype=torch.float16, device=device).permute(1, 2, 0)
        sfa, sfa_p = _uniform_scales(gen, l, m, sf_k, device)
        sfb, sfb_p = _uniform_scales(gen, l, 128, sf_k, device)
        return (a.view(FP4X2), b.permute(1, 2, 0).view(FP4X2), sfa, sfb, sfa_p, sfb_p, c)
    if problem == "gemm":
        a = _uniform_bytes(gen, (l, m, k // 2), device).permute(1, 2, 0)
        b = _uniform_bytes(gen, (l, n, k // 2), device).permute(1, 2, 0)
        c = torch.zeros((l, m, n), dtype=torch.float16, device=device).permute(1, 2, 0)
        sfa, sfa_p = _uniform_scales(gen, l, m, sf_k, device)
        sfb, sfb_p = _uniform_scales(gen, l, n, sf_k, device)
        return (a.view(FP4X2), b.view(FP4X2), sfa, sfb, sfa_p, sfb_p, c)
    if problem == "dual":
        a = _uniform_bytes(gen, (l, m, k // 2), device).permute(1, 2, 0)
        b1 = _uniform_bytes(gen, (l, n, k // 2), device).permute(1, 2, 0)
        b2 = _uniform_bytes(gen, (l, n, k // 2), device).permute(1, 2, 0)
        c = torch.zeros((l, m, n), dtype=torch.float16, device=device).permute(1, 2, 0)
        sfa, sfa_p = _uniform_scales(gen, l, m, sf_k, device)
        sfb1, sfb1_p = _uniform_scales(gen, l, n, sf_k, device)
        sfb2, sfb2_p = _uniform_scales(gen, l, n, sf_k, device)
        return (a.view(FP4X2), b1.view(FP4X2), b2.view(FP4X2), sfa, sfb1, sfb2,
                sfa_p, sfb1_p, sfb2_p, c)
    raise ValueError(problem)
