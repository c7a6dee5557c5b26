"""Regenerate the golden fixtures in this folder from the reference's own fixture files.

The reference (yipihey/GraphGP.jl) pins its refine path with JAX/Python-generated fixtures:
``test/reference/small.npz`` and ``medium.npz`` (written by ``test/dump_reference.py``) and
``test/reference/generate_parity.npz`` (written by ``test/python_parity_generate.py``), and its
anisotropic path with ``test/reference/aniso_parity.npz`` (``test/python_parity_aniso.py``).  This
script copies their arrays, unchanged, into compressed ``.npz`` files here so the tests can run
where the reference tree is absent (the GPU box).  Run it where the reference is mounted:

    python tests/golden/make_golden.py /path/to/GraphGP.jl
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
NAMES = ("small", "medium", "generate_parity", "aniso_parity")


def main(ref_root: str) -> None:
    for name in NAMES:
        src = os.path.join(ref_root, "test", "reference", f"{name}.npz")
        with np.load(src) as d:
            arrays = {k: d[k] for k in d.files}
        dst = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(dst, **arrays)
        print(f"{src} -> {dst} ({os.path.getsize(dst)} bytes, {len(arrays)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <GraphGP.jl checkout>")
    main(sys.argv[1])
