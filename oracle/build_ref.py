"""Build the reference's CUDA kernels (as a checker) into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.

    python oracle/build_ref.py [--reference <QVGGT checkout>]

Compiles, in place from the reference checkout (nothing is copied), the
kernel sources of the path:

    quantization_new/gemm/gemm_cuda.cu, quantization_new/gemv/gemv_cuda.cu,
    w8a8/w8a8_gemm_cuda.cu, w8a8/quantization.cu, w8a8/act.cu,
    w8a8/layernorm.cu, rope_new/fused_rope_with_pos.cu

plus this directory's ref_bind.cpp, with the reference's own nvcc flags
(``awq_inference_engine/setup.py:5-39``: -O3 --use_fast_math -DENABLE_BF16
and the half/bfloat16 operator macros) for sm_100a, into
``oracle/_ref/awq_ref*.so`` (a torch extension; its Ampere-era mma.sync /
ldmatrix / cp.async code is valid on sm_100).  The reference's own setup.py is
not used: it lists sources the reference does not ship.  Built files stay out
of git; they travel to the GPU box with the working tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")

SOURCES = [
    "quantization_new/gemm/gemm_cuda.cu",
    "quantization_new/gemv/gemv_cuda.cu",
    "w8a8/w8a8_gemm_cuda.cu",
    "w8a8/quantization.cu",
    "w8a8/act.cu",
    "w8a8/layernorm.cu",
    "rope_new/fused_rope_with_pos.cu",
]

NVCC_FLAGS = ["-O3", "-std=c++17", "-DENABLE_BF16", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
              "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
              "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_BFLOAT162_CONVERSIONS__", "--expt-relaxed-constexpr",
              "--expt-extended-lambda", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a"]


def built_path() -> str | None:
    if not os.path.isdir(OUT):
        return None
    for f in os.listdir(OUT):
        if f.startswith("awq_ref") and f.endswith(".so"):
            return os.path.join(OUT, f)
    return None


def load():
    """Import the built checker (raises ImportError if it was not built)."""
    p = built_path()
    if p is None:
        raise ImportError("oracle/_ref not built")
    import importlib.util
    spec = importlib.util.spec_from_file_location("awq_ref", p)
    mod = importlib.util.module_from_spec(spec)
    import torch  # noqa: F401  (the extension links against torch)
    spec.loader.exec_module(mod)
    return mod


def build(reference: str) -> str:
    csrc = os.path.join(reference, "qvggt", "runtime", "awq_inference_engine", "csrc")
    srcs = [os.path.join(csrc, s) for s in SOURCES]
    for s in srcs:
        if not os.path.exists(s):
            raise FileNotFoundError(s)
    os.makedirs(OUT, exist_ok=True)
    bdir = os.path.join(OUT, "build")
    os.makedirs(bdir, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load as tload
    tload(name="awq_ref", sources=[os.path.join(HERE, "ref_bind.cpp")] + srcs, build_directory=bdir,
          extra_cflags=["-O3", "-std=c++17", "-DENABLE_BF16"], extra_cuda_cflags=NVCC_FLAGS, verbose=False)
    so = [f for f in os.listdir(bdir) if f.startswith("awq_ref") and f.endswith(".so")][0]
    dst = os.path.join(OUT, so)
    shutil.copy2(os.path.join(bdir, so), dst)
    return dst


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference checkout (default: QVGGT_REFERENCE, else BASELINE.json's reference_path)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    if a.reference is None:
        sys.path.insert(0, os.path.dirname(HERE))
        from oracle.refpath import reference_path
        a.reference = reference_path()
    if not a.reference or not os.path.isdir(a.reference):
        print("reference checkout not present; oracle/_ref not built", file=sys.stderr)
        sys.exit(0)
    if built_path() is not None and not a.force:
        print(built_path())
        sys.exit(0)
    print(build(a.reference))
