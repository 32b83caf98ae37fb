"""Imports the reference's own NVFP4 modules from the baseline/_ref install.

Each problem directory of the reference (``problems/nvidia/nvfp4_*``) has
modules with the same top-level names (``reference``, ``task``, ``utils``,
``submission``) that import one another by those names.  ``load`` executes
one of them with its own problem directory first on ``sys.path`` and the
shared names cleared from ``sys.modules``, then restores the previous
entries, so the three problems' modules live side by side in one process
under private names.  Nothing here modifies the reference's files.

Used by the GPU parity tests (``generate_input``, ``ref_kernel``,
``check_implementation`` of ``nvfp4_*/reference.py``) and by ``bench.py
--suite`` (the reference's CuTe ``custom_kernel``s and ``ref_kernel``).
"""
from __future__ import annotations

import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.path.join(HERE, "_ref", "problems", "nvidia")
PROBLEM_DIRS = {"gemv": "nvfp4_gemv", "gemm": "nvfp4_gemm", "dual": "nvfp4_dual_gemm"}
_SHARED = ("task", "utils", "reference", "submission")
_LOADED: dict = {}


def available() -> bool:
    return all(os.path.isfile(os.path.join(REF_ROOT, d, "reference.py")) for d in PROBLEM_DIRS.values())


def problem_dir(problem: str) -> str:
    return os.path.join(REF_ROOT, PROBLEM_DIRS[problem])


def load(problem: str, module: str = "reference"):
    """The reference's ``<module>.py`` of ``problem`` ("gemv" | "gemm" | "dual")."""
    key = (problem, module)
    if key in _LOADED:
        return _LOADED[key]
    if not available():
        raise FileNotFoundError(f"reference not installed under {REF_ROOT} (run baseline/install_reference.py)")
    pdir = problem_dir(problem)
    path = os.path.join(pdir, module + ".py")
    saved = {n: sys.modules.pop(n) for n in _SHARED if n in sys.modules}
    # the GEMV problem has no utils.py of its own and uses problems/nvidia/utils.py
    extra = [pdir, REF_ROOT]
    sys.path[:0] = extra
    try:
        spec = importlib.util.spec_from_file_location(f"_nvfp4_ref_{problem}_{module}", path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[module] = mod
        spec.loader.exec_module(mod)
    finally:
        for n in _SHARED:
            sys.modules.pop(n, None)
        sys.modules.update(saved)
        del sys.path[:len(extra)]
    _LOADED[key] = mod
    return mod


def test_shapes(problem: str, section: str = "tests") -> list[dict]:
    """The ``tests:`` or ``benchmarks:`` list of the problem's task.yml."""
    import yaml
    with open(os.path.join(problem_dir(problem), "task.yml")) as f:
        return list(yaml.safe_load(f)[section])
