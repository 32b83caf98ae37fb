"""CPU tests of the oracle (no GPU): decode tables, the blocked scale layout,
known-answer products, and the golden fixtures produced on a B200 with
torch._scaled_mm (the reference's ref_kernel arithmetic)."""
import glob
import os

import numpy as np
import pytest
import torch

from nvfp4_b200 import inputs
from oracle import oracle

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def test_e2m1_table_matches_ocp_definition():
    # code = s e1 e0 m; value = (-1)^s * 2^(e-1) * (1 + m/2) for e > 0, m/2 for e == 0
    for code in range(16):
        s, e, m = code >> 3, (code >> 1) & 3, code & 1
        v = (m * 0.5) if e == 0 else 2.0 ** (e - 1) * (1 + m / 2)
        assert oracle.E2M1_VALUES[code] == (-v if s else v)


def test_e2m1_nibble_order():
    # byte 0x21: low nibble 1 (0.5) is element 0, high nibble 2 (1.0) element 1
    assert list(oracle.decode_e2m1(np.array([[0x21]], np.uint8))[0]) == [0.5, 1.0]


def test_e4m3_table_matches_torch():
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(np.isnan(t), np.isnan(oracle.E4M3FN_VALUES))
    ok = ~np.isnan(t)
    np.testing.assert_array_equal(t[ok], oracle.E4M3FN_VALUES[ok])


def test_e4m3_encoder_matches_torch():
    x = torch.empty(20000).uniform_(0.0, 450.0)
    x = torch.cat([x, -x, torch.tensor([0.25, 2.0, 1.0625, 0.0, 448.0])]).clamp(-448, 448)
    np.testing.assert_array_equal(oracle.encode_e4m3(x.numpy()), x.to(torch.float8_e4m3fn).view(torch.uint8).numpy())


@pytest.mark.parametrize("rows,sk", [(128, 4), (256, 16), (384, 448)])
def test_blocked_layout_roundtrip(rows, sk):
    rng = np.random.default_rng(rows + sk)
    plain = rng.integers(0, 256, size=(rows, sk), dtype=np.uint8)
    flat = oracle.to_blocked(plain)
    np.testing.assert_array_equal(oracle.from_blocked(flat, rows, sk), plain)
    # the torch restatement used by the drop-ins builds the same order
    np.testing.assert_array_equal(inputs.to_blocked(torch.from_numpy(plain)).numpy(), flat)


def test_reference_input_permuted_slots_equal_blocked_plain():
    d = inputs.reference_input("gemm", 256, 512, 2, 1111, n=128, device="cpu")
    sfa, sfa_p = d[2], d[4]
    for l in range(2):
        blk = sfa_p[..., l].permute(2, 4, 0, 1, 3).contiguous().view(torch.uint8).numpy().reshape(-1)
        np.testing.assert_array_equal(blk, oracle.to_blocked(sfa[:, :, l].view(torch.uint8).numpy()))


def test_known_answer_every_code_times_every_scale():
    # A row with code c in one group, scale s; b = all ones (code 2) with scale 1.0 (0x38).
    for c in range(16):
        for s in range(0, 127, 7):
            a = np.zeros((1, 8), np.uint8)
            a[0, 0] = c  # element 0 = code c, element 1..15 = 0
            sfa = np.array([[s]], np.uint8)
            b = np.full((1, 8), 0x22, np.uint8)
            sfb = np.array([[0x38]], np.uint8)
            got = oracle.gemm_f64(a, b, sfa, sfb)[0, 0]
            assert got == oracle.E2M1_VALUES[c] * oracle.E4M3FN_VALUES[s]


def test_known_answer_hand_summed_row():
    # 32 elements: a = +1.5 everywhere (code 3 -> byte 0x33), b alternates +6/-0.5 (codes 7, 9 -> 0x97)
    a = np.full((1, 16), 0x33, np.uint8)
    b = np.full((1, 16), 0x97, np.uint8)
    sfa = np.array([[0x38, 0x40]], np.uint8)  # 1.0, 2.0
    sfb = np.array([[0x30, 0x38]], np.uint8)  # 0.5, 1.0
    # group g: 8 * (1.5*6 + 1.5*-0.5) = 66 per group, scaled by sfa*sfb
    expect = 66 * 1.0 * 0.5 + 66 * 2.0 * 1.0
    assert oracle.gemm_f64(a, b, sfa, sfb)[0, 0] == expect


def test_silu_gate_overflow_to_inf_like_torch():
    x = np.array([20000.0, -20000.0, 3.0], np.float32)
    y = np.array([10.0, 10.0, 2.0], np.float32)
    got = oracle.silu_mul_f32(x, y).astype(np.float16)
    ref = (torch.nn.functional.silu(torch.from_numpy(x)) * torch.from_numpy(y)).to(torch.float16).numpy()
    np.testing.assert_array_equal(got, ref)


def test_mismatch_semantics_follow_verbose_allclose():
    e = np.array([1.0, np.inf, -np.inf, np.nan, 100.0])
    r = np.array([1.0025, np.inf, np.inf, np.nan, 100.2])
    bad = oracle.mismatches(r, e)
    assert list(bad) == [True, False, True, False, True]


@pytest.mark.skipif(not GOLDEN, reason="no golden fixtures")
@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_matches_scaled_mm_golden(path):
    z = np.load(path)
    out = z["out"]
    name = os.path.basename(path)
    m, n, l = out.shape
    got = np.empty_like(out)
    for i in range(l):
        if name.startswith("dual"):
            got[:, :, i] = oracle.ref_dual(z["a"][:, :, i], z["b1"][:, :, i], z["b2"][:, :, i],
                                           z["sfa"][:, :, i], z["sfb1"][:, :, i], z["sfb2"][:, :, i])
        elif name.startswith("gemv"):
            got[:, 0, i] = oracle.ref_gemv(z["a"][:, :, i], z["b"][:, :, i], z["sfa"][:, :, i], z["sfb"][:, :, i])
        else:
            got[:, :, i] = oracle.ref_gemm(z["a"][:, :, i], z["b"][:, :, i], z["sfa"][:, :, i], z["sfb"][:, :, i])
    assert not oracle.allclose_report(got, out), oracle.allclose_report(got, out)
    if not name.startswith("dual"):
        # single GEMMs: products are exact and fp32/f64 sums agree to the fp16 bit here
        np.testing.assert_array_equal(got, out)


def test_golden_inputs_match_reference_generator_on_cpu_shapes():
    # the fixtures were drawn on CUDA with the reference's RNG sequence; on CPU the
    # generator only has to reproduce shapes and value sets
    d = inputs.reference_input("dual", 128, 256, 1, 1111, n=128, device="cpu")
    a = d[0].view(torch.uint8)
    assert int((a & 0x44).max()) == 0  # nibbles keep only sign + 2 LSBs (0b1011)
