"""Host-only checks of the C ABI (no GPU): the library loads, exports every
function declared in include/nvfp4_b200.h, and rejects bad arguments with the
documented error codes before touching the device."""
import os
import re

import pytest

from nvfp4_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nvfp4_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(nvfp4_\w+)\s*\(", src, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared()
    assert set(names) >= {"nvfp4_gemv", "nvfp4_gemm", "nvfp4_dual_gemm", "nvfp4_last_error"}
    for n in names:
        assert hasattr(lib, n), n
    assert set(_lib.EXPORTS) <= set(names)
    assert lib.nvfp4_abi_version() == 1


FAKE = 1 << 20  # 16-byte aligned non-null pointer value; never dereferenced


def test_null_pointer_rejected():
    lib = _lib.load()
    rc = lib.nvfp4_gemm(None, FAKE, FAKE, FAKE, FAKE, 128, 128, 256, 1, 0, 0, 0, 0, 128, 0, None)
    assert rc == 3 and b"null" in lib.nvfp4_last_error()


@pytest.mark.parametrize("m,n,k", [(100, 128, 256), (128, 200, 256), (128, 128, 300), (0, 128, 256)])
def test_bad_gemm_shapes_rejected(m, n, k):
    lib = _lib.load()
    rc = lib.nvfp4_gemm(FAKE, FAKE, FAKE, FAKE, FAKE, m, n, k, 1, 0, 0, 0, 0, max(n, 1), 0, None)
    assert rc == 1, lib.nvfp4_last_error()
    with pytest.raises(_lib.Nvfp4Error):
        _lib.check(rc)


def test_misaligned_operand_rejected():
    lib = _lib.load()
    rc = lib.nvfp4_dual_gemm(FAKE + 8, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 128, 256, 1, 0, 0, 0, 0, 128, 0, None)
    assert rc == 2


def test_gemv_shape_checks():
    lib = _lib.load()
    assert lib.nvfp4_gemv(FAKE, FAKE, FAKE, FAKE, FAKE, 128, 100, 1, 0, 0, 0, 0, 0, None) == 1
    assert lib.nvfp4_gemv(FAKE, FAKE, FAKE, FAKE, FAKE, 130, 256, 1, 0, 0, 0, 0, 0, None) == 1
    assert lib.nvfp4_gemv(FAKE + 4, FAKE, FAKE, FAKE, FAKE, 128, 256, 1, 0, 0, 0, 0, 0, None) == 2


def test_ops_refuse_cpu_tensors():
    import torch
    from nvfp4_b200 import inputs, ops
    data = inputs.reference_input("gemm", 128, 256, 1, 1, n=128, device="cpu")
    with pytest.raises(_lib.Nvfp4Error, match="CUDA"):
        ops.gemm(data)
