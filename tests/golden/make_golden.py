"""Generates the golden fixtures under tests/golden/ on a CUDA B200.

For each case it imports the reference's own problems/nvidia/nvfp4_*/reference.py
from the baseline/_ref copy (baseline/install_reference.py, baseline/refload.py),
draws the inputs with its generate_input and computes the outputs with its
ref_kernel (torch._scaled_mm -> cuBLASLt).  Inputs (plain-layout bytes) and
the fp16 outputs are stored as .npz, with `meta` naming the reference files
and the library versions; tests/test_oracle.py checks the CPU oracle against
them without a GPU.

Usage (on a GPU box, with baseline/_ref installed):
    python tests/golden/make_golden.py --out tests/golden
"""
import argparse
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "reference-kernels_b200"))

sys.path.insert(0, os.path.join(ROOT, "baseline"))
import refload  # noqa: E402

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
    versions = f"torch {torch.__version__}, {torch.cuda.get_device_name(0)}, cuda {torch.version.cuda}"
    for problem, kw in CASES:
        kw = dict(kw)
        ref = refload.load(problem)
        src = f"problems/nvidia/{refload.PROBLEM_DIRS[problem]}/reference.py"
        meta = f"inputs: {src} generate_input{tuple(kw.items())}; out: {src} ref_kernel; {versions}"
        data = ref.generate_input(**kw)
        out = ref.ref_kernel(tuple(t.clone() for t in data))
        torch.cuda.synchronize()
        n = kw.pop("n", None)
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
