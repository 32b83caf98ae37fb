"""Parity of the sm_100a kernels (through the C ABI via the custom_kernel
drop-ins) against (1) the CPU oracle and (2) the reference's own arithmetic,
torch._scaled_mm, on identical seeded inputs.  Tolerance: rtol = atol = 1e-3,
the reference's check_implementation (problems/nvidia/*/reference.py)."""
import numpy as np
import pytest
import torch

from nvfp4_b200 import inputs, ops
from oracle import oracle
from tests.refcheck import assert_match, oracle_ref, scaled_mm_ref

pytestmark = pytest.mark.gpu

FN = {"gemv": ops.gemv, "gemm": ops.gemm, "dual": ops.dual_gemm}


def run(problem, data):
    out = FN[problem](data)
    torch.cuda.synchronize()
    from nvfp4_b200 import _lib
    assert _lib.device_status(True) == 0
    return out


# Shapes from the reference's task.yml `tests:` lists (seed 1111).
GEMV_TESTS = [(128, 256, 1), (128, 1536, 1), (128, 3072, 1), (256, 7168, 1), (2432, 4608, 2),
              (384, 7168, 2), (512, 512, 2), (512, 4096, 2), (512, 1536, 2)]
GEMM_TESTS = [(128, 256, 256), (128, 1536, 7168), (128, 3072, 1536), (256, 7168, 256), (256, 7168, 2048),
              (2304, 4608, 7168), (384, 7168, 2304), (512, 512, 7168), (512, 4096, 512), (512, 1536, 7168)]
DUAL_TESTS = [(1536, 512, 7168), (256, 512, 256), (3072, 1024, 1536), (7168, 1024, 256), (7168, 2304, 2048),
              (4608, 384, 7168), (7168, 384, 2304), (512, 768, 7168), (4096, 768, 512)]


@pytest.fixture(params=["tensorcore", "simt"])
def gemv_path(request, monkeypatch):
    """Both GEMV kernels: the TMA + tcgen05 one (default for K % 256 == 0) and the SIMT one."""
    if request.param == "simt":
        monkeypatch.setenv("NVFP4_GEMV_PATH", "simt")
    else:
        monkeypatch.delenv("NVFP4_GEMV_PATH", raising=False)
    return request.param


@pytest.mark.parametrize("m,k,l", GEMV_TESTS)
def test_gemv_reference_tests(m, k, l, gemv_path):
    data = inputs.reference_input("gemv", m, k, l, 1111)
    ref = scaled_mm_ref("gemv", data)
    out = run("gemv", data)
    assert_match(out, ref, f"gemv {m}x{k}x{l} vs _scaled_mm")


@pytest.mark.parametrize("m,n,k", GEMM_TESTS)
def test_gemm_reference_tests(m, n, k):
    data = inputs.reference_input("gemm", m, k, 1, 1111, n=n)
    ref = scaled_mm_ref("gemm", data)
    out = run("gemm", data)
    assert_match(out, ref, f"gemm {m}x{n}x{k} vs _scaled_mm")


@pytest.mark.parametrize("m,n,k", DUAL_TESTS)
def test_dual_reference_tests(m, n, k):
    data = inputs.reference_input("dual", m, k, 1, 1111, n=n)
    ref = scaled_mm_ref("dual", data)
    out = run("dual", data)
    assert_match(out, ref, f"dual {m}x{n}x{k} vs _scaled_mm")


# Small cases against the CPU oracle (both distributions, batched L).
@pytest.mark.parametrize("dist", ["reference", "baseline"])
@pytest.mark.parametrize("problem,m,n,k,l", [
    ("gemv", 256, 1, 1024, 3), ("gemv", 128, 1, 16384, 1), ("gemv", 512, 1, 2112, 2),
    ("gemm", 128, 128, 256, 1), ("gemm", 256, 384, 1024, 2), ("gemm", 384, 256, 2048, 1),
    ("dual", 128, 128, 256, 1), ("dual", 256, 256, 768, 2),
])
def test_against_oracle(dist, problem, m, n, k, l):
    gen = inputs.reference_input if dist == "reference" else inputs.baseline_input
    data = gen(problem, m, k, l, 7, n=None if problem == "gemv" else n)
    exp = oracle_ref(problem, data)
    out = run(problem, data)
    assert_match(out, exp, f"{problem} {m}x{n}x{k}x{l} ({dist}) vs oracle")


@pytest.mark.parametrize("m,k,l", [(7168, 16384, 4), (4096, 7168, 8), (7168, 2048, 4), (128, 1024, 1)])
def test_gemv_benchmark_shapes_and_repeat(m, k, l, gemv_path):
    """The reference's GEMV benchmark shapes (and configs[1]) on uniform inputs,
    called twice: split row blocks are combined deterministically."""
    data = inputs.baseline_input("gemv", m, k, l, 5)
    ref = scaled_mm_ref("gemv", data)
    o1 = run("gemv", data).clone()
    o2 = run("gemv", data).clone()
    assert torch.equal(o1, o2)
    assert_match(o1, ref, f"gemv {m}x{k}x{l} vs _scaled_mm")


def test_repeat_calls_identical():
    data = inputs.baseline_input("gemm", 256, 2048, 1, 3, n=256)
    o1 = run("gemm", data).clone()
    o2 = run("gemm", data).clone()
    assert torch.equal(o1, o2)


def test_non_contiguous_output_shard():
    """An N-shard written into a column slice of a wider C (the multi-GPU path)."""
    from nvfp4_b200 import _lib
    m, n, k = 256, 512, 1024
    a, b, sfa, sfb, sfa_p, sfb_p, c = inputs.baseline_input("gemm", m, k, 1, 5, n=n)
    full = ops.gemm((a, b, sfa, sfb, sfa_p, sfb_p, c)).clone()
    torch.cuda.synchronize()
    out = torch.zeros_like(c)
    lib = _lib.load()
    n0, n1 = 128, 384
    k2 = k // 2
    _lib.check(lib.nvfp4_gemm(a.data_ptr(), b.data_ptr() + n0 * k2, sfa_p.data_ptr(),
                              sfb_p.data_ptr() + (n0 // 128) * k * 8, out.data_ptr() + n0 * 2,
                              m, n1 - n0, k, 1, a.stride(2), b.stride(2), m * k // 16, n * k // 16,
                              out.stride(0), out.stride(2), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(out[:, n0:n1], full[:, n0:n1])
    assert torch.count_nonzero(out[:, :n0]) == 0 and torch.count_nonzero(out[:, n1:]) == 0


@pytest.mark.parametrize("splits", [2, 3, 5, 7])
@pytest.mark.parametrize("problem,m,n,k", [("gemm", 256, 512, 2816), ("dual", 256, 384, 2816), ("gemm", 128, 256, 1280),
                                           ("gemm", 128, 512, 3584)])
def test_split_k_matches_oracle_and_repeats(problem, m, n, k, splits, monkeypatch):
    """Split-K tiles (partials combined in split order by the last arriver):
    parity with the CPU oracle and bit-identical repeated calls."""
    monkeypatch.setenv("NVFP4_SPLITS", str(splits))
    data = inputs.baseline_input(problem, m, k, 1, 9, n=n)
    exp = oracle_ref(problem, data)
    o1 = run(problem, data).clone()
    o2 = run(problem, data).clone()
    assert torch.equal(o1, o2)
    assert_match(o1, exp, f"{problem} {m}x{n}x{k} splits={splits}")


@pytest.mark.parametrize("m,n,k", [(256, 4096, 7168), (512, 4096, 7168), (256, 3072, 4096), (512, 3072, 7168)])
def test_dual_benchmark_shapes(m, n, k):
    """The reference's dual-GEMM benchmark shapes (split K) against _scaled_mm."""
    data = inputs.reference_input("dual", m, k, 1, 1111, n=n)
    ref = scaled_mm_ref("dual", data)
    out = run("dual", data)
    assert_match(out, ref, f"dual {m}x{n}x{k} vs _scaled_mm")


@pytest.mark.parametrize("m,n,k,l", [(256, 256, 256, 1), (512, 1024, 2048, 1), (768, 512, 1024, 2), (2304, 4608, 7168, 1)])
def test_pair_gemm_matches_single_cta_and_oracle(m, n, k, l, monkeypatch):
    """2-CTA (cta_group::2, 256x256 tiles) GEMM against the 1-CTA kernel
    (bit-identical: same fp32 accumulation order per K step is not guaranteed,
    so the tolerance check is the gate) and the CPU oracle on small shapes."""
    monkeypatch.setenv("NVFP4_SPLITS", "1")
    data = inputs.baseline_input("gemm", m, k, l, 21, n=n)
    monkeypatch.setenv("NVFP4_PAIR", "0")
    single = run("gemm", data).clone()
    monkeypatch.setenv("NVFP4_PAIR", "1")
    pair1 = run("gemm", data).clone()
    pair2 = run("gemm", data).clone()
    assert torch.equal(pair1, pair2)
    assert_match(pair1, single, f"pair vs single {m}x{n}x{k}x{l}")
    if m * n * k <= 768 * 1024 * 2048:
        assert_match(pair1, oracle_ref("gemm", data), f"pair vs oracle {m}x{n}x{k}x{l}")


@pytest.mark.parametrize("form", ["hybrid", "pure"])
@pytest.mark.parametrize("kernel", ["single", "pair"])
@pytest.mark.parametrize("m,n,k,l", [
    (1664, 3072, 512, 1),    # 156 tiles of 128x256, ~2.1 K tiles per CTA: tiles cut three ways
    (1280, 2176, 1024, 1),   # N % 256 != 0: 128x128 tiles, 170 of them
    (1024, 7168, 2048, 1),   # benchmark config's M, N (224 tiles / 112 pair tiles), short K
    (768, 3328, 1280, 2),    # L = 2: ranges cross batch boundaries
    (2560, 4096, 512, 1),    # 160 pair tiles, ~4.3 K tiles per pair: pair tiles cut three ways
])
def test_stream_k_gemm(m, n, k, l, kernel, form, monkeypatch):
    """Stream-K GEMM (equal (tile, K tile) ranges per CTA or CTA pair, after
    whole-tile waves in the hybrid form; partial tiles combined through the
    workspace) against the oracle / _scaled_mm, the classic tile-per-worker
    path, and itself (bit-identical on repeat)."""
    if kernel == "pair" and (m % 256 or n % 256):
        pytest.skip("2-CTA tiles need M % 256 == 0 and N % 256 == 0")
    data = inputs.baseline_input("gemm", m, k, l, 33, n=n)
    monkeypatch.setenv("NVFP4_PAIR", "1" if kernel == "pair" else "0")
    monkeypatch.setenv("NVFP4_STREAMK", "-1")
    classic = run("gemm", data).clone()
    monkeypatch.setenv("NVFP4_STREAMK", "1" if form == "hybrid" else "2")
    sk1 = run("gemm", data).clone()
    sk2 = run("gemm", data).clone()
    assert torch.equal(sk1, sk2)
    assert_match(sk1, classic, f"stream-K vs classic {m}x{n}x{k}x{l}")
    if m * n * k * l <= 1664 * 3072 * 512:
        assert_match(sk1, oracle_ref("gemm", data), f"stream-K vs oracle {m}x{n}x{k}x{l}")
    else:
        assert_match(sk1, scaled_mm_ref("gemm", data), f"stream-K vs _scaled_mm {m}x{n}x{k}x{l}")


@pytest.mark.parametrize("kernel", ["single", "pair"])
@pytest.mark.parametrize("m,n,k", [(256, 512, 1024), (512, 384, 2048), (384, 512, 1024), (256, 4096, 7168)])
def test_dual_single_and_pair_kernels(m, n, k, kernel, monkeypatch):
    """Dual GEMM on the 1-CTA kernel (128 x (B1|B2) tiles, K split in
    clusters) and on the 2-CTA kernel (256 x (B1|B2) tiles, K split by
    stream-K ranges) against the oracle / _scaled_mm, repeated bit-identically."""
    if kernel == "pair" and m % 256:
        pytest.skip("2-CTA tiles need M % 256 == 0")
    monkeypatch.setenv("NVFP4_PAIR", "1" if kernel == "pair" else "0")
    data = inputs.baseline_input("dual", m, k, 1, 44, n=n)
    out1 = run("dual", data).clone()
    out2 = run("dual", data).clone()
    assert torch.equal(out1, out2)
    if m * n * k <= 512 * 512 * 2048:
        assert_match(out1, oracle_ref("dual", data), f"dual {kernel} {m}x{n}x{k} vs oracle")
    else:
        assert_match(out1, scaled_mm_ref("dual", data), f"dual {kernel} {m}x{n}x{k} vs _scaled_mm")


@pytest.mark.parametrize("problem,m,n,k", [("dual", 256, 128, 7168), ("dual", 256, 256, 2048), ("gemm", 256, 256, 7168)])
def test_pair_stream_k_many_contributors(problem, m, n, k, monkeypatch):
    """One or two tiles spread over many pairs (pure stream-K, up to ~10
    pairs per tile): the finaliser combines many partial slots."""
    monkeypatch.setenv("NVFP4_PAIR", "1")
    monkeypatch.setenv("NVFP4_STREAMK", "2")
    data = inputs.baseline_input(problem, m, k, 1, 55, n=n)
    out1 = run(problem, data).clone()
    out2 = run(problem, data).clone()
    assert torch.equal(out1, out2)
    assert_match(out1, oracle_ref(problem, data), f"{problem} {m}x{n}x{k} many contributors vs oracle")


@pytest.mark.parametrize("kernel", ["single", "pair", "streamk"])
@pytest.mark.parametrize("problem,m,n,k,l", [
    ("gemm", 256, 256, 64, 1), ("gemm", 256, 512, 192, 2), ("gemm", 512, 512, 320, 1), ("gemm", 256, 768, 1856, 1),
    ("gemm", 2048, 2560, 320, 1),  # 160 tiles: no K split, so the 2-CTA kernel runs under "pair"
    ("gemm", 1664, 3072, 320, 1),  # 156 tiles: stream-K ranges (under "streamk") over a partial last K tile
    ("dual", 256, 256, 448, 1), ("dual", 512, 384, 1344, 1),
])
def test_k_tail(problem, m, n, k, l, kernel, monkeypatch):
    """K % 256 != 0 (K % 64 == 0): a partial last K tile issues only its
    remaining 64-wide MMA steps and copies only their scale blocks; checked
    on the 1-CTA kernel (with its K-split clusters), the pair kernel and
    stream-K against the oracle."""
    monkeypatch.setenv("NVFP4_PAIR", "1" if kernel == "pair" else "0")
    if kernel == "streamk":
        if problem == "dual":
            pytest.skip("stream-K is a GEMM option")
        monkeypatch.setenv("NVFP4_STREAMK", "2")
        monkeypatch.setenv("NVFP4_PAIR", "0")
    data = inputs.baseline_input(problem, m, k, l, 66, n=n)
    out = run(problem, data).clone()
    assert_match(out, oracle_ref(problem, data), f"{problem} {kernel} {m}x{n}x{k}x{l} K tail vs oracle")


def test_workspace_growth_inside_capture_is_refused_then_works_uncaptured():
    """A call that would have to grow the library's per-device workspace
    inside a CUDA-graph capture returns an error before enqueuing anything
    (the capture stays valid); the same call outside a capture grows the
    workspace and is correct, and then captures and replays correctly."""
    from nvfp4_b200 import _lib
    m, k, l = 128 * 4096, 256, 4  # 16384 row blocks: a 16 MB workspace, larger than any other test's
    data = inputs.baseline_input("gemv", m, k, l, 8)
    ops._CACHE.clear()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        with pytest.raises(_lib.Nvfp4Error, match="stream capture"):
            ops.gemv(data)
    torch.cuda.synchronize()
    out = run("gemv", data).clone()
    assert_match(out, scaled_mm_ref("gemv", data), "gemv after workspace growth")
    data[-1].zero_()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        ops.gemv(data)
    g2.replay()
    torch.cuda.synchronize()
    assert torch.equal(data[-1], out)


@pytest.mark.parametrize("m,k,l", [(128, 64, 1), (128, 192, 3), (256, 256, 8), (128, 320, 2), (384, 16384 + 256, 1)])
def test_gemv_edges_against_oracle(m, k, l, gemv_path):
    """GEMV edge cases: the smallest K (one 64-element scale group of four),
    K that is not a multiple of 256 (SIMT kernel), many batches, and K one
    256-wide tile past a power of two (the tensor-core kernel's partial last
    unit), on both kernels where they apply, against the CPU oracle."""
    data = inputs.baseline_input("gemv", m, k, l, 17)
    out = run("gemv", data)
    assert_match(out, oracle_ref("gemv", data), f"gemv {m}x{k}x{l}")


@pytest.mark.parametrize("problem,m,n,k,l", [("gemm", 512, 512, 1024, 2), ("dual", 512, 256, 1024, 3)])
def test_pair_kernel_batched(problem, m, n, k, l, monkeypatch):
    """2-CTA tiles over several batch indices (tiles of every batch in one
    persistent launch) against the CPU oracle."""
    monkeypatch.setenv("NVFP4_PAIR", "1")
    data = inputs.baseline_input(problem, m, k, l, 23, n=n)
    out = run(problem, data)
    assert_match(out, oracle_ref(problem, data), f"{problem} pair {m}x{n}x{k}x{l}")


def test_dual_output_shard_through_the_c_abi():
    """A dual-GEMM N-shard written through offset B1/B2/scale/C pointers and
    the full problem's ldc (the multi-GPU path) equals the same columns of
    the whole problem; columns outside the shard stay untouched."""
    from nvfp4_b200 import _lib
    m, n, k = 256, 512, 1024
    a, b1, b2, sfa, sfb1, sfb2, sfa_p, sfb1_p, sfb2_p, c = inputs.baseline_input("dual", m, k, 1, 29, n=n)
    full = ops.dual_gemm((a, b1, b2, sfa, sfb1, sfb2, sfa_p, sfb1_p, sfb2_p, c)).clone()
    torch.cuda.synchronize()
    out = torch.zeros_like(c)
    n0, n1 = 256, 512
    k2 = k // 2
    lib = _lib.load()
    _lib.check(lib.nvfp4_dual_gemm(a.data_ptr(), b1.data_ptr() + n0 * k2, b2.data_ptr() + n0 * k2, sfa_p.data_ptr(),
                                   sfb1_p.data_ptr() + (n0 // 128) * k * 8, sfb2_p.data_ptr() + (n0 // 128) * k * 8,
                                   out.data_ptr() + n0 * 2, m, n1 - n0, k, 1, a.stride(2), b1.stride(2),
                                   m * k // 16, n * k // 16, out.stride(0), out.stride(2),
                                   torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(out[:, n0:n1], full[:, n0:n1])
    assert torch.count_nonzero(out[:, :n0]) == 0
