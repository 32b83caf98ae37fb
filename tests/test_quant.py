"""NVFP4 quantiser and scale-layout converter: CPU known-answer tests of the
oracle, and (GPU) bit-exact parity of the CUDA kernels with it, layout round
trips, and quantise -> custom_kernel end to end."""
import numpy as np
import pytest
import torch

from nvfp4_b200 import inputs, ops
from oracle import oracle
from tests.refcheck import assert_match, oracle_ref, u8


def test_e2m1_encoder_ties_to_even_and_saturates():
    x = np.array([0, .2, .25, .3, .74, .75, 1.25, 1.26, 1.75, 2.5, 2.6, 3.5, 5, 5.1, 1e9, -0.1, -7], np.float32)
    want = [0, 0, 0, 1, 1, 2, 2, 3, 4, 4, 5, 6, 6, 7, 7, 8, 15]
    assert list(oracle.encode_e2m1(x)) == want


def test_e2m1_encoder_inverts_decoder():
    codes = np.arange(16, dtype=np.uint8)
    assert list(oracle.encode_e2m1(oracle.E2M1_VALUES[codes])) == list(codes)


def test_quantize_known_block():
    # amax 6.5 -> s = 6.5/6 -> e4m3 1.125 (code 0x39); x / 1.125 rounded to e2m1
    x = np.array([[0, .2, .25, .3, .75, 1.25, 1.75, 2.5, 3.5, 5, 5.1, -.1, -6.5, 1, 2, 3]], np.float32)
    packed, codes = oracle.quantize(x)
    assert codes.tolist() == [[0x39]]
    deq = oracle.dequant(packed, codes)[0]
    assert np.all(np.abs(deq - x[0]) <= 0.5 * 1.125 * 2 + 1e-6)  # within half the coarsest e2m1 step x scale


def test_quantize_zero_and_saturation():
    x = np.zeros((1, 32), np.float32)
    x[0, 16:] = 1e6  # amax / 6 > 448 saturates the scale, values saturate to 6
    packed, codes = oracle.quantize(x)
    assert codes[0, 0] == 0 and codes[0, 1] == 0x7E
    assert np.all(packed[0, :8] == 0) and np.all(packed[0, 8:] == 0x77)




def _rand(rows, k, l, dtype, scale, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((l, rows, k), generator=g, device="cuda", dtype=torch.float32) * scale
    x[:, :, :16] = 0  # an all-zero block in every row
    return x.to(dtype).permute(1, 2, 0)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("scale,gs", [(1.0, 1.0), (1e-3, 1.0), (3000.0, 1.0), (5.0, 0.03125)])
def test_quantize_matches_oracle_bit_exact(dtype, scale, gs):
    from nvfp4_b200 import quant
    x = _rand(256, 1024, 2, dtype, scale, 3)
    packed, perm = quant.quantize(x, gs)
    torch.cuda.synchronize()
    for l in range(2):
        want_p, want_s = oracle.quantize(x[:, :, l].float().cpu().numpy(), gs)
        np.testing.assert_array_equal(u8(packed[:, :, l]), want_p)
        blk = perm[..., l].permute(2, 4, 0, 1, 3).contiguous().view(torch.uint8).cpu().numpy().reshape(-1)
        np.testing.assert_array_equal(blk, oracle.to_blocked(want_s))


@pytest.mark.gpu
def test_scale_layout_roundtrip_and_matches_reference_order():
    from nvfp4_b200 import quant
    d = inputs.reference_input("gemm", 384, 2048, 3, 11, n=128)
    sfa, sfa_p = d[2], d[4]
    blk = quant.to_blocked(sfa)
    torch.cuda.synchronize()
    assert torch.equal(blk.view(torch.uint8), sfa_p.view(torch.uint8))
    assert blk.stride() == sfa_p.stride()
    plain = quant.to_plain(sfa_p)
    assert torch.equal(plain.view(torch.uint8), sfa.view(torch.uint8))


@pytest.mark.gpu
@pytest.mark.parametrize("problem", ["gemm", "dual"])
def test_quantize_then_custom_kernel(problem):
    """Quantised real data feeds custom_kernel directly; the result equals the
    oracle on the quantised operands and approximates the fp32 product."""
    from nvfp4_b200 import quant
    m, n, k = 256, 256, 1024
    xa = _rand(m, k, 1, torch.bfloat16, 1.0, 5)
    xb = _rand(n, k, 1, torch.bfloat16, 1.0, 6)
    xb2 = _rand(n, k, 1, torch.bfloat16, 1.0, 7)
    a, sa = quant.quantize(xa)
    b, sb = quant.quantize(xb)
    c = torch.empty((1, m, n), dtype=torch.float16, device="cuda").permute(1, 2, 0)
    if problem == "gemm":
        data = (a, b, quant.to_plain(sa), quant.to_plain(sb), sa, sb, c)
    else:
        b2, sb2 = quant.quantize(xb2)
        data = (a, b, b2, quant.to_plain(sa), quant.to_plain(sb), quant.to_plain(sb2), sa, sb, sb2, c)
    fn = ops.gemm if problem == "gemm" else ops.dual_gemm
    out = fn(data)
    torch.cuda.synchronize()
    assert_match(out, oracle_ref(problem, data), f"quantised {problem}")
    if problem == "gemm":
        exact = (xa[:, :, 0].float() @ xb[:, :, 0].float().T)
        rel = (out[:, :, 0].float() - exact).norm() / exact.norm()
        assert rel < 0.15, rel  # NVFP4 quantisation error of both operands
