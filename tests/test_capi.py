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
    assert lib.nvfp4_abi_version() == 2


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


def test_packed_forms_reject_like_the_scalar_forms():
    """The *_call entry points take the same arguments in one struct and
    return the same codes."""
    import ctypes
    lib = _lib.load()
    assert lib.nvfp4_gemm_call(None) == 3
    g = _lib.GemmArgs(FAKE, FAKE, None, FAKE, FAKE, None, FAKE, 100, 128, 256, 1, 0, 0, 0, 0, 128, 0, None)
    assert lib.nvfp4_gemm_call(ctypes.byref(g)) == 1
    g.M, g.a = 128, FAKE + 8
    assert lib.nvfp4_gemm_call(ctypes.byref(g)) == 2
    g.a, g.b2, g.sfb2_blk = FAKE, FAKE + 8, FAKE
    assert lib.nvfp4_dual_gemm_call(ctypes.byref(g)) == 2
    v = _lib.GemvArgs(FAKE, FAKE, FAKE, FAKE, FAKE, 130, 256, 1, 0, 0, 0, 0, 0, 0, None)
    assert lib.nvfp4_gemv_call(ctypes.byref(v)) == 1


def test_packed_struct_layout_matches_header(tmp_path):
    """Field offsets of the ctypes mirrors equal those the C compiler gives the
    header's structs."""
    import ctypes
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    fields = {"nvfp4_gemv_args": _lib.GemvArgs, "nvfp4_gemm_args": _lib.GemmArgs}
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in fields.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l}
    for cname, py in fields.items():
        assert got[(cname, "size")] == ctypes.sizeof(py)
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
