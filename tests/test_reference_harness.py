"""The drop-ins under the reference's real evaluation harness.

For each problem a scratch directory is laid out the way the competition
runner lays it out: the harness script (problems/nvidia/eval_better_bench.py
for the GEMM and dual GEMM, problems/nvidia/eval.py for the GEMV), the
problem's reference.py and task.py and the shared utils.py, all unmodified
from the baseline/_ref install, plus this build's drop-in as submission.py.
The harness runs as its own process with POPCORN_FD on a pipe, in ``test``
mode on several task.yml test shapes and in ``benchmark`` mode on one
benchmark shape; the test parses the ``key: value`` lines it writes
(eval_better_bench.py:452-506, eval.py:429-485)."""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline"))
import refload  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refload.available(), reason="reference not installed in baseline/_ref")]

HARNESS = {"gemv": "eval.py", "gemm": "eval_better_bench.py", "dual": "eval_better_bench.py"}
SUBMISSION = {"gemv": "nvfp4_gemv", "gemm": "nvfp4_gemm", "dual": "nvfp4_dual_gemm"}


def _spec_line(spec):
    return "; ".join(f"{k}: {v}" for k, v in spec.items())


def _run_harness(tmp_path, problem, mode, specs, timeout=900):
    d = tmp_path / f"{problem}_{mode}"
    d.mkdir()
    pdir = refload.problem_dir(problem)
    shutil.copyfile(os.path.join(refload.REF_ROOT, HARNESS[problem]), d / HARNESS[problem])
    shutil.copyfile(os.path.join(refload.REF_ROOT, "utils.py"), d / "utils.py")
    for name in ("reference.py", "task.py"):
        shutil.copyfile(os.path.join(pdir, name), d / name)
    shutil.copyfile(os.path.join(ROOT, "reference-kernels_b200", "submissions", SUBMISSION[problem], "submission.py"),
                    d / "submission.py")
    (d / "cases.txt").write_text("\n".join(_spec_line(s) for s in specs) + "\n")
    rfd, wfd = os.pipe()
    env = dict(os.environ, POPCORN_FD=str(wfd), NVFP4_B200_HOME=os.path.join(ROOT, "reference-kernels_b200"))
    proc = subprocess.Popen([sys.executable, HARNESS[problem], mode, "cases.txt"], cwd=d, env=env,
                            pass_fds=(wfd,), stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    os.close(wfd)
    with os.fdopen(rfd) as f:
        report = f.read()
    out, _ = proc.communicate(timeout=timeout)
    kv = {}
    for line in report.splitlines():
        if ": " in line:
            key, val = line.split(": ", 1)
            kv[key.strip()] = val.strip()
    return proc.returncode, kv, report, out.decode(errors="replace")[-3000:]


@pytest.mark.parametrize("problem", ["gemv", "gemm", "dual"])
def test_harness_test_mode(tmp_path, problem):
    specs = refload.test_shapes(problem, "tests")[:4]
    rc, kv, report, log = _run_harness(tmp_path, problem, "test", specs)
    assert kv.get("check") == "pass", f"rc={rc}\n{report}\n{log}"
    assert kv.get("test-count") == str(len(specs))
    for i in range(len(specs)):
        assert kv.get(f"test.{i}.status") == "pass", report


@pytest.mark.parametrize("problem", ["gemv", "gemm", "dual"])
def test_harness_benchmark_mode(tmp_path, problem):
    specs = refload.test_shapes(problem, "benchmarks")[:1]
    rc, kv, report, log = _run_harness(tmp_path, problem, "benchmark", specs)
    assert rc == 0, f"rc={rc}\n{report}\n{log}"
    assert kv.get("benchmark-count") == "1", report
    mean_ns = float(kv["benchmark.0.mean"])
    assert 0 < mean_ns < 1e6, report
    print(f"{problem} {specs[0]}: harness mean {mean_ns / 1e3:.2f} us")
