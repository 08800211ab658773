"""Build the reference's own CUDA optimizer extension as a test-only checker.

TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Nothing under the product package may
import what this script produces.

The reference ships its FP8 AdamW step as five C++/CUDA files
(coat/optimizer/kernels/{bindings.cpp, fp8_adamw_cuda.cpp,
fp8_adamw_cuda_kernel.cu, fp8_adamw_expand_cuda.cpp,
fp8_adamw_expand_cuda_kernel.cu}).  This recipe compiles those files where
they lie in the reference checkout (no source is copied) with nvcc for
sm_100a and writes the resulting python module ``qoptim_cuda`` into
``oracle/_ref/`` (git-ignored; it travels to the GPU machine as a built
file).  The GPU parity tests load it, when present, as the bit-level checker
for the fused optimizer kernels.

Usage:  python oracle/build_ref.py [/path/to/reference]
"""
import os
import sys


def build(reference_root="/root/reference", verbose=False):
    here = os.path.dirname(os.path.abspath(__file__))
    out = os.path.join(here, "_ref")
    src = os.path.join(reference_root, "coat", "optimizer", "kernels")
    names = ["bindings.cpp", "fp8_adamw_cuda.cpp", "fp8_adamw_cuda_kernel.cu",
             "fp8_adamw_expand_cuda.cpp", "fp8_adamw_expand_cuda_kernel.cu"]
    sources = [os.path.join(src, n) for n in names]
    if not all(os.path.exists(s) for s in sources):
        return None
    os.makedirs(out, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load
    # same nvcc options as the reference's setup.py (-O3, C++17, no fast-math)
    load(name="qoptim_cuda", sources=sources, build_directory=out,
         extra_cuda_cflags=["-O3", "-std=c++17",
                            "-gencode", "arch=compute_100a,code=sm_100a"],
         extra_cflags=["-O3", "-std=c++17"],
         is_python_module=False, verbose=verbose)
    so = os.path.join(out, "qoptim_cuda.so")
    return so if os.path.exists(so) else None


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    print(build(root, verbose=True))
