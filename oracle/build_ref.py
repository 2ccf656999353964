"""Build the reference's own CUDA kernel for sm_100a into oracle/_ref/ (TEST INFRASTRUCTURE ONLY).

The reference's only native code is the group-128 GEMV ``gemv_g128_v2`` and its host wrapper,
kept as the string ``CUDA_SRC`` in experiments/speed_fair_kaggle.py:656-692 and compiled there
with ``torch.utils.cpp_extension.load_inline`` (:695-696).  This recipe reads that string from
the reference checkout where it lies (nothing is copied into this repository), and makes the
same ``load_inline`` call with ``-gencode arch=compute_100a,code=sm_100a`` and the build
directory ``oracle/_ref/``.  The resulting extension module ``exact_gemv_ref`` is what
``tests/test_gpu_ref_kernel.py`` runs beside ``exb_gemv`` (same outputs, and the B200 timing of
both kernels).  The product never loads it.

Usage:  python oracle/build_ref.py [--ref <reference checkout>]
"""
import argparse
import ast
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
SRC_REL = "experiments/speed_fair_kaggle.py"
CPP_DECL = "torch::Tensor gemv(torch::Tensor x, torch::Tensor wT, torch::Tensor Mg);"   # speed_fair_kaggle.py:695


def reference_cuda_source(ref):
    """The value of the module-level assignment CUDA_SRC = r\"\"\"...\"\"\" of the reference script."""
    with open(os.path.join(ref, SRC_REL)) as f:
        tree = ast.parse(f.read())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "CUDA_SRC" for t in node.targets):
            return ast.literal_eval(node.value)
    raise RuntimeError(f"CUDA_SRC not found in {SRC_REL}")


def build(ref="/root/reference", verbose=False):
    if not os.path.isdir(ref):
        return None
    from torch.utils.cpp_extension import load_inline
    os.makedirs(OUT, exist_ok=True)
    return load_inline(name="exact_gemv_ref", cpp_sources=CPP_DECL, cuda_sources=reference_cuda_source(ref),
                       functions=["gemv"], build_directory=OUT, verbose=verbose, with_cuda=True,
                       extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"])


def load():
    """Import the built module (no compiler involved); None if it was not built."""
    path = os.path.join(OUT, "exact_gemv_ref.so")
    if not os.path.exists(path):
        return None
    import importlib.util
    import torch  # noqa: F401  (the extension links against torch's libraries)
    spec = importlib.util.spec_from_file_location("exact_gemv_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    a = ap.parse_args()
    if build(a.ref, verbose=True) is None:
        sys.exit(f"reference checkout not found at {a.ref}")
    print("built", os.path.join(OUT, "exact_gemv_ref.so"))
