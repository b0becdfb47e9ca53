"""Build recipe for the reference's own CUDA extension (test infrastructure).

The reference's fused Wan Q/K/V producer (``src/sparsepr/kernels/n8_ext/csrc/
n8_ops.cu``, a single-file PyTorch extension) is compiled here directly from
the reference checkout with the flags of the reference's own CMake recipe
(``n8_ext/CMakeLists.txt``: fast math, relaxed constexpr, extended lambdas),
for sm_100a, into ``oracle/_ref/n8_ext/n8_kernels.so`` (git-ignored; the built
module travels with the repository snapshot to a GPU box, where the reference
checkout does not exist).  It serves only as a checker: ``tests/golden/
make_wan_qkv_golden.py`` runs it on a GPU to record reference outputs.

    python -m oracle.build_ref            # build (needs the reference checkout)
"""

from __future__ import annotations

import importlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_BUILD = os.path.join(HERE, "_ref", "n8_ext")


def reference_root() -> str | None:
    """The reference checkout next to this repository, if present."""
    root = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    src = os.path.join(root, "src", "sparsepr", "kernels", "n8_ext", "csrc", "n8_ops.cu")
    return root if os.path.exists(src) else None


def build(force: bool = False) -> str | None:
    """Compile the reference extension; returns the .so path (None without the reference)."""
    root = reference_root()
    so = os.path.join(REF_BUILD, "n8_kernels.so")
    if root is None:
        return so if os.path.exists(so) else None
    src = os.path.join(root, "src", "sparsepr", "kernels", "n8_ext", "csrc", "n8_ops.cu")
    if os.path.exists(so) and not force and os.path.getmtime(so) >= os.path.getmtime(src):
        return so
    from torch.utils.cpp_extension import load

    os.makedirs(REF_BUILD, exist_ok=True)
    load(name="n8_kernels", sources=[src], build_directory=REF_BUILD, verbose=False,
         extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a", "--use_fast_math",
                            "--expt-relaxed-constexpr", "--expt-extended-lambda", "--disable-warnings"],
         extra_cflags=["-w"], with_cuda=True)
    return so


def load_reference_kernels():
    """Import the prebuilt reference extension module (``n8_kernels``)."""
    if REF_BUILD not in sys.path:
        sys.path.insert(0, REF_BUILD)
    return importlib.import_module("n8_kernels")


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
