"""Parity against the reference's OWN code, imported unmodified from the
baseline/_ref install (baseline/install_reference.py, baseline/refload.py):

* inputs come from the reference's ``generate_input``
  (problems/nvidia/nvfp4_*/reference.py) for every ``tests:`` and
  ``benchmarks:`` shape of its task.yml;
* the drop-in ``custom_kernel`` gets a fresh clone of each input, as the
  reference harness does (eval_better_bench.py:221-238), and its output is
  judged by the reference's ``check_implementation`` (rtol = atol = 1e-3 with
  the nan / inf checks of utils.py:30-95), which runs ``ref_kernel``
  (torch._scaled_mm) itself;
* BASELINE.json configs 1-4 (uniform bytes, scales uniform in [0.25, 2]) are
  judged the same way;
* the build's restatement of ``generate_input`` (nvfp4_b200.inputs) is
  checked bit-exact against the reference's.
"""
import os
import sys

import pytest
import torch

from nvfp4_b200 import _lib, inputs, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline"))
import refload  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refload.available(),
                                 reason="reference not installed: python baseline/install_reference.py --src <ref>")]

FN = {"gemv": ops.gemv, "gemm": ops.gemm, "dual": ops.dual_gemm}


def _clone(data):
    return tuple(t.clone() if isinstance(t, torch.Tensor) else t for t in data)


def _check(problem, data, what):
    ref = refload.load(problem)
    out = FN[problem](_clone(data))
    torch.cuda.synchronize()
    assert _lib.device_status(True) == 0, f"{what}: device status set"
    ok, msg = ref.check_implementation(_clone(data), out)
    assert ok, f"{what}: {msg}"
    return out


def _cases(section):
    out = []
    for problem in ("gemv", "gemm", "dual"):
        if not refload.available():
            continue
        for spec in refload.test_shapes(problem, section):
            out.append(pytest.param(problem, spec, id=f"{problem}-" + "-".join(f"{k}{v}" for k, v in spec.items())))
    return out


@pytest.mark.parametrize("problem,spec", _cases("tests"))
def test_reference_tests(problem, spec):
    data = refload.load(problem).generate_input(**spec)
    _check(problem, data, f"{problem} {spec}")


@pytest.mark.parametrize("problem,spec", _cases("benchmarks"))
def test_reference_benchmarks(problem, spec):
    """Benchmark shapes with several of the seeds the harness derives from
    them (seed + 42 i, eval_better_bench.py:180-183)."""
    gen = refload.load(problem).generate_input
    for i in (1, 2, 50):
        s = dict(spec, seed=spec["seed"] + 42 * i)
        _check(problem, gen(**s), f"{problem} {s}")


BASELINE_CONFIGS = [("gemv", 7168, 1, 16384, 4, 1), ("gemm", 1024, 7168, 16384, 1, 2),
                    ("dual", 256, 4096, 7168, 1, 3), ("gemm", 16384, 16384, 16384, 1, 4)]


@pytest.mark.parametrize("problem,m,n,k,l,idx", BASELINE_CONFIGS, ids=[f"config{c[-1]}" for c in BASELINE_CONFIGS])
def test_baseline_configs(problem, m, n, k, l, idx):
    """BASELINE.json configs 1-4 at full size, through the default kernel
    choice (config 2 runs the 2-CTA pair kernel over 64 K tiles)."""
    data = inputs.baseline_input(problem, m, k, l, 1111 + idx, n=None if problem == "gemv" else n)
    out1 = _check(problem, data, f"config {idx}")
    out2 = FN[problem](_clone(data))
    torch.cuda.synchronize()
    assert torch.equal(out1, out2), f"config {idx}: repeated call differs"


@pytest.mark.parametrize("problem,spec", [
    ("gemv", dict(m=256, k=1024, l=2, seed=1111)), ("gemv", dict(m=128, k=7168, l=1, seed=77)),
    ("gemm", dict(m=256, n=384, k=512, l=2, seed=1111)), ("gemm", dict(m=128, n=7168, k=2048, l=1, seed=1153)),
    ("dual", dict(m=256, n=128, k=768, l=1, seed=1111)), ("dual", dict(m=128, n=256, k=256, l=2, seed=9)),
])
def test_generate_input_restatement_is_bit_exact(problem, spec):
    """nvfp4_b200.inputs.reference_input replays generate_input's RNG calls;
    every tensor it returns equals the reference's, byte for byte, in the
    same shape and strides."""
    ref = refload.load(problem).generate_input(**spec)
    kw = dict(spec)
    mine = inputs.reference_input(problem, kw.pop("m"), kw.pop("k"), kw.pop("l"), kw.pop("seed"), n=kw.pop("n", None))
    assert len(ref) == len(mine)
    for i, (r, x) in enumerate(zip(ref, mine)):
        assert r.shape == x.shape and r.stride() == x.stride(), f"slot {i}: {r.shape}/{r.stride()} vs {x.shape}/{x.stride()}"
        assert r.dtype == x.dtype, f"slot {i}: {r.dtype} vs {x.dtype}"
        if r.dtype == torch.float16:
            assert torch.equal(r, x), f"slot {i} differs"
        else:
            assert torch.equal(r.view(torch.uint8), x.view(torch.uint8)), f"slot {i} differs"
