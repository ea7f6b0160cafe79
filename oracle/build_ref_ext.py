"""Build the reference's own CUDA extension from its sources, for B200.

TEST INFRASTRUCTURE ONLY: the result is a checker and a timing baseline for
tests/test_gpu_reference_ext.py; the product never loads it.

    MASK_LOSS_REF=<reference checkout> python oracle/build_ref_ext.py

Compiles src/bindings.cpp, src/cpu/matching.cpp and src/cuda/*.cu of the
reference where they lie (nothing is copied), with the reference's own nvcc
flags (setup.py:31-38 of AndyBarcia/mask_loss) for sm_100, into
oracle/_ref/ext/ (ignored by git; it travels to the GPU box with the other
built files).  The module is the reference's ``mask_loss`` extension with the
11 ops of src/bindings.cpp:157-169.  Without the reference checkout the build
is skipped.
"""
from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "ext")


def build(verbose: bool = False):
    # run as a script, this directory would shadow the package of the same name
    sys.path[:] = [q for q in sys.path if os.path.abspath(q or ".") != HERE]
    sys.path.insert(0, os.path.dirname(HERE))
    from oracle.oracle import reference_root

    root = reference_root()
    if root is None:
        print("reference checkout not found (MASK_LOSS_REF): skipping the reference extension")
        return None
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    src = os.path.join(root, "src")
    sources = (glob.glob(os.path.join(src, "*.cpp")) + glob.glob(os.path.join(src, "cpu", "*.cpp")) +
               sorted(glob.glob(os.path.join(src, "cuda", "*.cu"))))
    os.makedirs(OUT, exist_ok=True)
    return load(
        name="mask_loss",
        sources=sources,
        extra_include_paths=[src],
        extra_cflags=["-O3", "-DWITH_CUDA"],
        extra_cuda_cflags=["-DWITH_CUDA", "-DCUDA_HAS_FP16=1", "-D__CUDA_NO_HALF_OPERATORS__",
                           "-D__CUDA_NO_HALF_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
                           "--use_fast_math", "-O3"],
        build_directory=OUT,
        verbose=verbose,
    )


def strip_objects() -> None:
    """Drop the object files (only the module travels; a rebuild recompiles)."""
    for f in glob.glob(os.path.join(OUT, "*.o")):
        os.remove(f)


if __name__ == "__main__":
    m = build(verbose="-v" in sys.argv)
    if m is not None:
        strip_objects()
    print("built" if m is not None else "skipped", OUT)
