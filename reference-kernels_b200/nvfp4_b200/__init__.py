"""B200 (sm_100a) NVFP4 GEMV / GEMM / dual GEMM behind the reference's
``custom_kernel(data) -> output`` plugin API (problems/nvidia/*/submission.py).

The kernels live in ``libnvfp4_b200.so`` (C ABI: include/nvfp4_b200.h), loaded
with ctypes by ``_lib``; ``ops`` holds the drop-in ``custom_kernel`` functions.
"""
from . import _lib, inputs, ops  # noqa: F401
from .ops import dual_gemm, gemm, gemv  # noqa: F401
