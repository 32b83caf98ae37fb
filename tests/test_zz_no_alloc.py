"""GPU test of nvfp4_gemv_noalloc, the GEMV entry point that allocates nothing.

It serves callers that cannot allocate device memory when they call the GEMV
(memory reserved up front by a pool or arena, host code without cudaMalloc):
the kernel's scratch lives in a fixed array inside the library.  The output
is checked against the regular entry point, nvfp4_gemv, and against the
reference's own arithmetic (torch._scaled_mm, as ref_kernel calls it) with
the reference's tolerance, rtol = atol = 1e-3.  This file is named so that
pytest collects it last; it must pass alone in a fresh process and after the
other tests (which leave the shared array and the regular workspace in
whatever state their last call left them).
"""
import pytest
import torch

from nvfp4_b200 import _lib, inputs, ops
from tests.refcheck import assert_match, scaled_mm_ref

pytestmark = pytest.mark.gpu


def _noalloc_into(data, out):
    a, b, _, _, sfa_p, sfb_p, c = data
    m, k2, l = a.shape
    lib = _lib.load()
    _lib.check(lib.nvfp4_gemv_noalloc(
        a.data_ptr(), b.data_ptr(), sfa_p.data_ptr(), sfb_p.data_ptr(), out.data_ptr(),
        m, 2 * k2, l, a.stride(2), b.stride(2), sfa_p.stride(5), sfb_p.stride(5), out.stride(2),
        torch.cuda.current_stream().cuda_stream))
    return out


def _noalloc(data):
    return _noalloc_into(data, torch.full_like(data[-1], float("nan")))


@pytest.mark.parametrize("m,k,l", [(7168, 16384, 4), (384, 7168, 2), (128, 256, 1)])
def test_noalloc_matches_gemv_on_two_calls(m, k, l, monkeypatch):
    monkeypatch.delenv("NVFP4_GEMV_PATH", raising=False)
    for seed in (11, 12):  # two calls in a row, on different inputs
        data = inputs.baseline_input("gemv", m, k, l, seed)
        want = ops.gemv(data).clone()
        got = _noalloc(data)
        torch.cuda.synchronize()
        assert _lib.device_status(True) == 0
        assert_match(got, want, f"noalloc vs nvfp4_gemv {m}x{k}x{l} seed {seed}")
        assert_match(got, scaled_mm_ref("gemv", data), f"noalloc vs _scaled_mm {m}x{k}x{l} seed {seed}")


def test_noalloc_back_to_back_without_sync_and_allocates_nothing():
    """Two no-alloc calls on different inputs into two outputs, issued back
    to back on one stream with one synchronisation at the end; the device's
    free memory is the same before and after a run of calls on a shape this
    process has not used before."""
    d1 = inputs.baseline_input("gemv", 2304, 7168, 3, 21)
    d2 = inputs.baseline_input("gemv", 2304, 7168, 3, 22)
    o1 = torch.full_like(d1[-1], float("nan"))
    o2 = torch.full_like(d2[-1], float("nan"))
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _noalloc_into(d1, o1)
        _noalloc_into(d2, o2)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert _lib.device_status(True) == 0
    assert_match(o1, scaled_mm_ref("gemv", d1), "noalloc back-to-back call 1")
    assert_match(o2, scaled_mm_ref("gemv", d2), "noalloc back-to-back call 2")


def test_noalloc_rejects_oversize_and_bad_shapes():
    lib = _lib.load()
    fake = 1 << 20
    # K % 256 != 0 is outside this entry point (the SIMT kernel needs no scratch)
    assert lib.nvfp4_gemv_noalloc(fake, fake, fake, fake, fake, 128, 320, 1, 0, 0, 0, 0, 0, None) == 1
    torch.cuda.init()
    # more 128-row blocks than the fixed array has arrival counters
    rc = lib.nvfp4_gemv_noalloc(fake, fake, fake, fake, fake, 128 * 16384, 256, 2, 0, 0, 0, 0, 0, None)
    assert rc == 1
    assert b"arrival counters" in lib.nvfp4_last_error()
    # partial sums that do not fit: 16384 blocks, each split over several SMs
    rc = lib.nvfp4_gemv_noalloc(fake, fake, fake, fake, fake, 128 * 8192, 16384 * 4, 2, 0, 0, 0, 0, 0, None)
    assert rc == 1
    assert b"bytes of scratch" in lib.nvfp4_last_error()
