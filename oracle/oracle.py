"""CPU oracle for the three NVFP4 problems (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The CUDA extension never falls back to it.

It restates, in numpy, what the reference computes for the hot path:

* ``ref_kernel`` of ``problems/nvidia/nvfp4_gemv/reference.py:28-54``,
  ``problems/nvidia/nvfp4_gemm/reference.py:27-53`` and
  ``problems/nvidia/nvfp4_dual_gemm/reference.py:27-77``: for every batch
  index ``l`` the product (A * sfA) @ (B * sfB)^T with fp32 (here: float64)
  accumulation, cast to fp16; the dual problem applies ``silu(x) * y`` in fp32
  before the cast (``nvfp4_dual_gemm/reference.py:76``).
* ``to_blocked`` of ``nvfp4_gemm/reference.py:12-24`` (the 128x4 scale-factor
  block layout that cuBLASLt and the "permuted" tuple slots use).
* ``verbose_allclose`` of ``problems/nvidia/utils.py:30-95`` (rtol/atol test
  with nan / +inf / -inf exclusive-or).

The reference's arithmetic itself lives in ``torch._scaled_mm`` (cuBLASLt,
closed source, torch 2.11.0+cu128), which cannot run on a CPU.  The decode
tables below follow the published OCP MX / NVFP4 definitions: e2m1 is
sign | 2-bit exponent (bias 1) | 1-bit mantissa, two codes per byte with the
element of even K index in the low nibble; e4m3fn is sign | 4-bit exponent
(bias 7) | 3-bit mantissa with 0x7f / 0xff as NaN and no infinities.
Parity of this restatement against ``torch._scaled_mm`` is pinned by the
golden fixtures under ``tests/golden/`` (generated on a B200 by
``tests/golden/make_golden.py``) and by the hand-derived known-answer tests in
``tests/test_oracle.py``.
"""
from __future__ import annotations

import numpy as np

SF_VEC = 16  # elements per block scale (reference.py: ``sf_vec_size = 16``)

# e2m1 magnitudes for codes 0..7; bit 3 is the sign.
_E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
E2M1_VALUES = np.concatenate([_E2M1_MAG, -_E2M1_MAG]).astype(np.float32)


def _make_e4m3fn_table() -> np.ndarray:
    t = np.empty(256, dtype=np.float32)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            t[code] = np.nan
        elif e == 0:
            t[code] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3FN_VALUES = _make_e4m3fn_table()

# byte -> (value of low nibble, value of high nibble)
_PAIR_TABLE = np.stack(
    [E2M1_VALUES[np.arange(256) & 0xF], E2M1_VALUES[np.arange(256) >> 4]], axis=1
).astype(np.float32)


def decode_e2m1(packed: np.ndarray) -> np.ndarray:
    """[..., K/2] uint8 -> [..., K] float32 (element 2j = low nibble of byte j)."""
    packed = np.asarray(packed, dtype=np.uint8)
    out = _PAIR_TABLE[packed]  # [..., K/2, 2]
    return out.reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def decode_e4m3(codes: np.ndarray) -> np.ndarray:
    return E4M3FN_VALUES[np.asarray(codes, dtype=np.uint8)]


def encode_e4m3(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> e4m3fn code (finite inputs, |x| <= 448)."""
    values = np.asarray(values, dtype=np.float32)
    finite = E4M3FN_VALUES.copy()
    finite[np.isnan(finite)] = np.inf
    pos = np.arange(128)  # codes 0..127 ascending, 127 is NaN
    pv = finite[:127]
    mag = np.abs(values)
    idx = np.searchsorted(pv, mag)  # pv[idx-1] < mag <= pv[idx]
    idx = np.clip(idx, 1, 126)
    lo, hi = pv[idx - 1], pv[idx]
    pick_hi = (hi - mag < mag - lo) | ((hi - mag == mag - lo) & ((idx & 1) == 0))
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(mag >= pv[126], 126, code)
    code = np.where(mag <= 0, 0, code)
    sign = (np.signbit(values) & (code != 0)).astype(np.uint8) << 7
    return (pos[code].astype(np.uint8) | sign).astype(np.uint8)


def encode_e2m1(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even, saturating fp32 -> e2m1 code (sign kept, also for zero)."""
    v = np.asarray(values, dtype=np.float32)
    mag = np.abs(v)
    # ties go to the even code: 0.25->0, 0.75->1.0, 1.25->1.0, 1.75->2, 2.5->2, 3.5->4, 5->4
    code = np.select(
        [mag <= 0.25, mag < 0.75, mag <= 1.25, mag < 1.75, mag <= 2.5, mag < 3.5, mag <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    return code | (np.signbit(v).astype(np.uint8) << 3)


def quantize(x: np.ndarray, global_scale: float = 1.0):
    """NVFP4 quantisation of x [rows, K] (values as float32): per 16-element
    block s = e4m3_rn_satfinite(amax / (6 g)), q = e2m1_rn_satfinite(x / (s g)),
    q = 0 where s decodes to 0.  Returns (packed [rows, K/2] uint8 with the even
    element in the low nibble, plain scale codes [rows, K/16] uint8).  Mirrors
    the producer step of generate_input (nvfp4_gemm/reference.py:56-158) for
    real data; divisions are IEEE fp32 round-to-nearest."""
    x = np.asarray(x, dtype=np.float32)
    rows, k = x.shape
    g = np.float32(global_scale)
    blocks = x.reshape(rows, k // SF_VEC, SF_VEC)
    amax = np.abs(blocks).max(axis=2)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        s = (amax / (np.float32(6.0) * g)).astype(np.float32)
    codes = encode_e4m3(np.minimum(s, np.float32(448.0)))
    d = (E4M3FN_VALUES[codes] * g).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        y = (blocks / d[:, :, None]).astype(np.float32)
    q = encode_e2m1(y)
    q = np.where(d[:, :, None] > 0, q, np.uint8(0)).reshape(rows, k)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return packed, codes.astype(np.uint8)


def dequant(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """packed [rows, K/2] uint8 and e4m3 codes [rows, K/16] -> float32 [rows, K]."""
    vals = decode_e2m1(packed)
    rows, k = vals.shape
    sf = decode_e4m3(scales)
    assert sf.shape == (rows, k // SF_VEC), (sf.shape, rows, k)
    return (vals.reshape(rows, k // SF_VEC, SF_VEC) * sf[:, :, None]).reshape(rows, k)


# ---------------------------------------------------------------------------
# scale-factor layouts (reference.py:12-24 and generate_input's permuted copy)
# ---------------------------------------------------------------------------

def blocked_offset(i: np.ndarray, j: np.ndarray, sk: int) -> np.ndarray:
    """Byte offset of plain scale (row i, column j) inside the 128x4 blocked layout."""
    return ((i // 128) * (sk // 4) * 512 + (j // 4) * 512 + (i % 32) * 16
            + ((i % 128) // 32) * 4 + (j % 4))


def to_blocked(plain: np.ndarray) -> np.ndarray:
    """[rows, SK] -> flat blocked vector (rows % 128 == 0, SK % 4 == 0)."""
    rows, sk = plain.shape
    assert rows % 128 == 0 and sk % 4 == 0, (rows, sk)
    out = np.empty(rows * sk, dtype=plain.dtype)
    i, j = np.meshgrid(np.arange(rows), np.arange(sk), indexing="ij")
    out[blocked_offset(i, j, sk).ravel()] = plain.ravel()
    return out


def from_blocked(flat: np.ndarray, rows: int, sk: int) -> np.ndarray:
    i, j = np.meshgrid(np.arange(rows), np.arange(sk), indexing="ij")
    return np.asarray(flat).reshape(-1)[blocked_offset(i, j, sk)]


# ---------------------------------------------------------------------------
# ref_kernel restatements.  All operands are per-batch numpy arrays in the
# plain layouts: a [M, K/2] uint8, b [N, K/2] uint8, sfa [M, K/16] uint8 codes,
# sfb [N, K/16] uint8 codes.  Results are float64 before the final cast.
# ---------------------------------------------------------------------------

def gemm_f64(a, b, sfa, sfb) -> np.ndarray:
    """(A*sfA) @ (B*sfB)^T in float64 (products of e2m1 x e4m3 are exact)."""
    da = dequant(a, sfa).astype(np.float64)
    db = dequant(b, sfb).astype(np.float64)
    return da @ db.T


def ref_gemm(a, b, sfa, sfb) -> np.ndarray:
    """nvfp4_gemm/reference.py:27-53 for one batch index: fp16 [M, N]."""
    return gemm_f64(a, b, sfa, sfb).astype(np.float32).astype(np.float16)


def ref_gemv(a, b_row, sfa, sfb_row) -> np.ndarray:
    """nvfp4_gemv/reference.py:28-54 for one batch index: fp16 [M] (column 0)."""
    return ref_gemm(a, b_row[:1], sfa, sfb_row[:1])[:, 0]


def silu_mul_f32(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    y = y.astype(np.float32)
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))) * y


def ref_dual(a, b1, b2, sfa, sfb1, sfb2) -> np.ndarray:
    """nvfp4_dual_gemm/reference.py:27-77 for one batch index: fp16 [M, N]."""
    r1 = gemm_f64(a, b1, sfa, sfb1).astype(np.float32)
    r2 = gemm_f64(a, b2, sfa, sfb2).astype(np.float32)
    with np.errstate(over="ignore"):
        return silu_mul_f32(r1, r2).astype(np.float16)


# ---------------------------------------------------------------------------
# tolerance check (utils.py:30-95)
# ---------------------------------------------------------------------------

def mismatches(received: np.ndarray, expected: np.ndarray, rtol=1e-3, atol=1e-3) -> np.ndarray:
    """Boolean mask of elements that verbose_allclose would report."""
    r = np.asarray(received, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert r.shape == e.shape, (r.shape, e.shape)
    with np.errstate(invalid="ignore"):
        tol = np.abs(r - e) > atol + rtol * np.abs(e)
    nan = np.isnan(r) ^ np.isnan(e)
    pinf = np.isposinf(r) ^ np.isposinf(e)
    ninf = np.isneginf(r) ^ np.isneginf(e)
    return tol | nan | pinf | ninf


def allclose_report(received, expected, rtol=1e-3, atol=1e-3, max_print=5) -> list[str]:
    bad = mismatches(received, expected, rtol, atol)
    n = int(bad.sum())
    if n == 0:
        return []
    idx = np.argwhere(bad)[:max_print]
    lines = [f"Number of mismatched elements: {n}"]
    for ix in idx:
        t = tuple(int(v) for v in ix)
        lines.append(f"ERROR AT {t}: {np.asarray(received)[t]} {np.asarray(expected)[t]}")
    return lines


# ---------------------------------------------------------------------------
# CPU port of ref_kernel for timing (bench.py's cpu_baseline and reference
# arm only): dequantise through the 256-entry byte -> (lo, hi) table and the
# e4m3 table into fp32, then an fp32 matmul, multithreaded through torch's
# CPU kernels -- the arithmetic of reference.py (dequantise to fp32, fp32
# GEMM, fp16 cast), run on host cores.
# ---------------------------------------------------------------------------

def torch_dequant(packed, scales):
    """packed [rows, K/2] uint8 tensor, scales [rows, K/16] uint8 codes -> fp32 [rows, K]."""
    import torch
    rows, k2 = packed.shape
    vals = torch.from_numpy(_PAIR_TABLE)[packed.long()].reshape(rows, 2 * k2)
    sf = torch.from_numpy(E4M3FN_VALUES)[scales.long()]
    return (vals.view(rows, -1, SF_VEC) * sf.unsqueeze(-1)).view(rows, 2 * k2)


def cpu_port(problem: str, a, b, sfa, sfb, b2=None, sfb2=None):
    """One batch index on the CPU: a/b/b2 packed uint8, sf* plain uint8 codes -> fp16."""
    import torch
    da = torch_dequant(a, sfa)
    if problem == "gemv":
        return (da @ torch_dequant(b[:1], sfb[:1])[0]).to(torch.float16)
    r1 = da @ torch_dequant(b, sfb).T
    if problem == "gemm":
        return r1.to(torch.float16)
    r2 = da @ torch_dequant(b2, sfb2).T
    return (torch.nn.functional.silu(r1) * r2).to(torch.float16)
