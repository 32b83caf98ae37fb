"""GPU test of nvfp4_gemv_noalloc, the GEMV entry point that allocates nothing.

It serves callers that cannot allocate device memory when they call the GEMV
(memory reserved up front by a pool or arena, host code without cudaMalloc):
the kernel's scratch lives in a fixed array inside the library.  This file is
named so that pytest collects it last; it must pass alone in a fresh process
and after the other tests (which leave the shared array and the regular
workspace in whatever state their last call left them).
"""
import pytest
import torch

from nvfp4_b200 import _lib, inputs, ops
from tests.refcheck import assert_match

pytestmark = pytest.mark.gpu


def _noalloc(data):
    a, b, _, _, sfa_p, sfb_p, c = data
    m, k2, l = a.shape
    out = torch.full_like(c, float("nan"))
    lib = _lib.load()
    _lib.check(lib.nvfp4_gemv_noalloc(
        a.data_ptr(), b.data_ptr(), sfa_p.data_ptr(), sfb_p.data_ptr(), out.data_ptr(),
        m, 2 * k2, l, a.stride(2), b.stride(2), sfa_p.stride(5), sfb_p.stride(5), out.stride(2),
        torch.cuda.current_stream().cuda_stream))
    return out


@pytest.mark.parametrize("m,k,l", [(7168, 16384, 4), (384, 7168, 2), (128, 256, 1)])
def test_noalloc_matches_gemv_on_two_calls(m, k, l, monkeypatch):
    monkeypatch.delenv("NVFP4_GEMV_PATH", raising=False)
    for seed in (11, 12):  # two calls in a row, on different inputs
        data = inputs.baseline_input("gemv", m, k, l, seed)
        want = ops.gemv(data).clone()
        got = _noalloc(data)
        torch.cuda.synchronize()
        assert_match(got, want, f"noalloc gemv {m}x{k}x{l} seed {seed}")


def test_noalloc_rejects_oversize_and_bad_shapes():
    lib = _lib.load()
    fake = 1 << 20
    # K % 256 != 0 is outside this entry point (the SIMT kernel needs no scratch)
    assert lib.nvfp4_gemv_noalloc(fake, fake, fake, fake, fake, 128, 320, 1, 0, 0, 0, 0, 0, None) == 1
    # a shape whose scratch need is larger than the fixed array
    torch.cuda.init()
    rc = lib.nvfp4_gemv_noalloc(fake, fake, fake, fake, fake, 128 * 16384, 256, 2, 0, 0, 0, 0, 0, None)
    assert rc == 1
    assert b"scratch" in lib.nvfp4_last_error() or b"needs" in lib.nvfp4_last_error()
