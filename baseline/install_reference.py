"""Installs the reference's NVFP4 problems, unmodified, into baseline/_ref.

The reference (SwayamInSync/reference-kernels) is plain Python on top of
torch / cuBLASLt / CuTe-DSL with no package metadata, so ``pip install
--target`` has nothing to build; the install is a byte-for-byte copy of
``problems/nvidia`` (the three problems' reference.py, task.py, task.yml,
utils.py, submission.py, template*.py and the two eval harnesses) into the
git-ignored ``baseline/_ref/problems/nvidia``.  The copy travels with the
repository snapshot to a GPU box, where the tests and ``bench.py --suite``
import ``generate_input`` / ``ref_kernel`` / ``check_implementation`` and the
reference's CuTe kernels from it (``baseline/refload.py``).  A manifest with
each file's sha256 is written beside it.

    python baseline/install_reference.py --src <reference checkout>
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")
SUBTREE = os.path.join("problems", "nvidia")


def install(src: str) -> dict:
    src_tree = os.path.join(src, SUBTREE)
    if not os.path.isdir(src_tree):
        raise SystemExit(f"{src_tree} not found")
    dst_tree = os.path.join(DEST, SUBTREE)
    if os.path.isdir(DEST):
        shutil.rmtree(DEST)
    files = {}
    for dirpath, _dirs, names in os.walk(src_tree):
        for name in sorted(names):
            if not name.endswith((".py", ".yml", ".yaml")):
                continue
            s = os.path.join(dirpath, name)
            rel = os.path.relpath(s, src_tree)
            d = os.path.join(dst_tree, rel)
            os.makedirs(os.path.dirname(d), exist_ok=True)
            shutil.copyfile(s, d)
            with open(d, "rb") as f:
                files[rel] = hashlib.sha256(f.read()).hexdigest()
    manifest = {"source": os.path.abspath(src), "subtree": SUBTREE, "files": files}
    with open(os.path.join(DEST, "MANIFEST.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    return manifest


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", required=True, help="root of a SwayamInSync/reference-kernels checkout")
    args = ap.parse_args(argv)
    m = install(args.src)
    print(f"installed {len(m['files'])} files into {os.path.join(DEST, SUBTREE)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
