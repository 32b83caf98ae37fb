"""Generates the golden fixtures under tests/golden/ on a CUDA B200.

For each case it draws the reference's own inputs (nvfp4_b200.inputs.reference_input,
which replays the RNG calls of problems/nvidia/*/reference.py:generate_input
on the CUDA device, so the tensors equal the reference's for that seed) and
computes ref_kernel through torch._scaled_mm exactly as
problems/nvidia/*/reference.py does.  Inputs (plain-layout bytes) and the
fp16 outputs are stored as .npz; tests/test_oracle.py checks the CPU oracle
against them without a GPU.

Usage (on a GPU box):  python tests/golden/make_golden.py --out tests/golden
"""
import argparse
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "reference-kernels_b200"))

from nvfp4_b200 import inputs  # noqa: E402
from tests.refcheck import scaled_mm_ref  # noqa: E402

CASES = [
    ("gemv", dict(m=128, k=256, l=1, seed=1111)),
    ("gemv", dict(m=256, k=1024, l=2, seed=1111)),
    ("gemm", dict(m=128, n=256, k=256, l=1, seed=1111)),
    ("gemm", dict(m=128, n=128, k=768, l=2, seed=1112)),
    ("dual", dict(m=256, n=128, k=256, l=1, seed=1111)),
    ("dual", dict(m=128, n=128, k=512, l=1, seed=1113)),
]


def u8(t):
    return t.view(torch.uint8).cpu().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(ROOT, "tests", "golden"))
    args = ap.parse_args()
    os.makedirs(args.out, exist_ok=True)
    meta = f"torch {torch.__version__}, {torch.cuda.get_device_name(0)}, cuda {torch.version.cuda}"
    for problem, kw in CASES:
        kw = dict(kw)
        n = kw.pop("n", None)
        data = inputs.reference_input(problem, n=n, device="cuda", **kw)
        out = scaled_mm_ref(problem, data)
        torch.cuda.synchronize()
        if problem == "dual":
            a, b1, b2, sfa, sfb1, sfb2 = data[:6]
            arrays = dict(a=u8(a), b1=u8(b1), b2=u8(b2), sfa=u8(sfa), sfb1=u8(sfb1), sfb2=u8(sfb2))
        else:
            a, b, sfa, sfb = data[:4]
            if problem == "gemv":
                b, sfb = b[:1], sfb[:1]
            arrays = dict(a=u8(a), b=u8(b), sfa=u8(sfa), sfb=u8(sfb))
        name = f"{problem}_m{kw['m']}_n{n or 1}_k{kw['k']}_l{kw['l']}_s{kw['seed']}.npz"
        np.savez_compressed(os.path.join(args.out, name), out=out.cpu().numpy(), meta=np.array(meta), **arrays)
        print("wrote", name, tuple(out.shape))


if __name__ == "__main__":
    main()
