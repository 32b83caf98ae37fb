"""The drop-in submission.py files used the way the reference harness uses a
submission (problems/nvidia/eval_better_bench.py:141-172, 214-274): the file
is copied into a flat working directory and imported as the module
``submission``; custom_kernel is called on deep clones of generate_input's
tuple (clone() keeps the permuted strides), on 50 inputs with distinct seeds,
and every output is checked with the reference's tolerance against
torch._scaled_mm (ref_kernel's arithmetic).  It needs no copy of the
reference; tests/test_reference_harness.py runs the reference's real harness."""
import importlib.util
import os
import shutil
import sys

import pytest
import torch

from nvfp4_b200 import inputs
from tests.refcheck import assert_match, scaled_mm_ref

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SUBS = os.path.join(ROOT, "reference-kernels_b200", "submissions")


def _clone(data):
    return tuple(t.clone() for t in data)


def _load_submission(problem_dir, tmp_path, monkeypatch):
    work = tmp_path / problem_dir
    work.mkdir()
    shutil.copy(os.path.join(SUBS, problem_dir, "submission.py"), work / "submission.py")
    monkeypatch.setenv("NVFP4_B200_HOME", os.path.join(ROOT, "reference-kernels_b200"))
    monkeypatch.syspath_prepend(str(work))
    sys.modules.pop("submission", None)
    spec = importlib.util.spec_from_file_location("submission", work / "submission.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("problem_dir,problem,shape", [
    ("nvfp4_gemv", "gemv", dict(m=4096, k=7168, l=2)),
    ("nvfp4_gemm", "gemm", dict(m=128, n=4096, k=7168, l=1)),
    ("nvfp4_dual_gemm", "dual", dict(m=256, n=3072, k=4096, l=1)),
])
@pytest.mark.gpu
def test_submission_module_like_the_harness(problem_dir, problem, shape, tmp_path, monkeypatch):
    mod = _load_submission(problem_dir, tmp_path, monkeypatch)
    assert mod.compile_kernel() is None
    shape = dict(shape)
    n = shape.pop("n", None)
    seed = 1111
    datas = []
    for _ in range(50):
        seed += 42
        datas.append(inputs.reference_input(problem, n=n, seed=seed, **shape))
    check = [_clone(d) for d in datas]
    outs = [mod.custom_kernel(_clone(d)) for d in datas]   # obligatory correctness pass
    torch.cuda.synchronize()
    for d, o in zip(check, outs):
        assert_match(o, scaled_mm_ref(problem, d), f"{problem_dir} submission")
    outs = [mod.custom_kernel(d) for d in datas]            # timed-loop form: same objects, not cloned
    torch.cuda.synchronize()
    for d, o in zip(check, outs):
        assert_match(o, scaled_mm_ref(problem, d), f"{problem_dir} submission (repeat)")
