"""Build the reference's own CUDA extension (csrc/w4a16_gemv.cu + csrc/bindings.cpp)
for sm_100a, from the sources where they lie in the reference checkout, into
oracle/_ref/ — TEST / COMPARISON INFRASTRUCTURE ONLY, never part of the product.

The reference builds this module with setuptools (setup.py:11-18); this recipe
compiles the same two files directly with torch.utils.cpp_extension (no use of
the reference's build system) so that its kernel can be timed on a B200 beside
focal_b200's.  The output is a plain torch extension module that exports the
reference's ``w4a16_linear(x, wq, scales, zeros)``.

    FOCAL_REFERENCE_DIR=<reference checkout> python oracle/build_ref_ext.py
    python oracle/build_ref_ext.py <reference checkout>

The checkout is given explicitly (argument or FOCAL_REFERENCE_DIR; there is no
default location).  The GPU machines do not have it and use the built .so.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "focal_w4a16_ref_C"


def build(ref_root: str) -> Path:
    from torch.utils.cpp_extension import load

    src = Path(ref_root) / "csrc"
    OUT.mkdir(exist_ok=True)
    load(name=NAME, sources=[str(src / "bindings.cpp"), str(src / "w4a16_gemv.cu")],
         extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
         extra_cflags=["-O3"], build_directory=str(OUT), verbose=False)
    return OUT / f"{NAME}.so"


def load_built():
    """Import the built module (torch must be importable; CUDA at call time)."""
    import torch  # noqa: F401  (loads the libraries the module links against)

    path = OUT / f"{NAME}.so"
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    import os

    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FOCAL_REFERENCE_DIR")
    if not root:
        sys.exit("give the reference checkout as an argument or in FOCAL_REFERENCE_DIR")
    print(build(root))
