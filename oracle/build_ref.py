"""Stage the reference's own implementation as a test-only checker.

TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Nothing under the product package may
import what this script produces.

Two things are produced, both into ``oracle/_ref/`` (git-ignored: nothing of the
reference enters this repository's history; the directory travels to the GPU
machine as built files):

1. ``qoptim_cuda.so``: the reference ships its FP8 AdamW step as five C++/CUDA
   files (coat/optimizer/kernels/{bindings.cpp, fp8_adamw_cuda.cpp,
   fp8_adamw_cuda_kernel.cu, fp8_adamw_expand_cuda.cpp,
   fp8_adamw_expand_cuda_kernel.cu}).  They are compiled where they lie in the
   reference checkout with nvcc for sm_100a.  The GPU parity tests load the
   module as the bit-level checker of the fused optimizer kernels.

2. ``coat_ref/``: an importable staging of the reference's python operator layer
   (coat/activation/real_quantization/*.py, the Triton kernels and their
   wrappers; coat/activation/liger/*.py, the loss head; coat/optimizer/fp8_adamw.py
   with the one configuration class it imports).  The files are byte-for-byte the reference's; only the package
   root is renamed so that it cannot shadow, or be shadowed by, anything else.
   The module that drags in plotting and model code (fp8linear.py) is left out.
   On a GPU the parity tests run these Triton kernels next to the CUDA kernels
   of this repository on the same tensors.

Usage:  python oracle/build_ref.py [/path/to/reference]
        (or COAT_REFERENCE_ROOT=/path/to/reference; without either, a checkout
        named ``reference`` beside this repository is used if there is one)
"""
import os
import shutil
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(_HERE, "_ref")

_STAGED = {
    # reference directory -> (destination under coat_ref/, file filter)
    ("coat", "activation", "real_quantization"): (("activation", "real_quantization"),
                                                  lambda n: n.endswith(".py") and n != "fp8linear.py"),
    ("coat", "activation", "liger"): (("activation", "liger"), lambda n: n.endswith(".py")),
    ("coat", "optimizer"): (("optimizer",), lambda n: n == "fp8_adamw.py"),
    ("coat", "utils"): (("utils",), lambda n: n == "_fp8_quantization_config.py"),
}


def reference_root(explicit=None):
    """Where the reference checkout is: argument, environment, or a sibling directory of this repository."""
    cands = [explicit, os.environ.get("COAT_REFERENCE_ROOT"),
             os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "coat")):
            return os.path.abspath(c)
    return None


def stage_python(root=None):
    """Copy the reference's operator-layer python files into oracle/_ref/coat_ref/ (see the module docstring)."""
    root = reference_root(root)
    if root is None:
        return None
    dst_root = os.path.join(OUT, "coat_ref")
    for src_parts, (dst_parts, keep) in _STAGED.items():
        src = os.path.join(root, *src_parts)
        dst = os.path.join(dst_root, *dst_parts)
        os.makedirs(dst, exist_ok=True)
        for name in sorted(os.listdir(src)):
            if keep(name):
                shutil.copyfile(os.path.join(src, name), os.path.join(dst, name))
    return dst_root


def build(root=None, verbose=False):
    """Compile the reference's optimizer extension into oracle/_ref/qoptim_cuda.so."""
    root = reference_root(root)
    if root is None:
        return None
    src = os.path.join(root, "coat", "optimizer", "kernels")
    names = ["bindings.cpp", "fp8_adamw_cuda.cpp", "fp8_adamw_cuda_kernel.cu",
             "fp8_adamw_expand_cuda.cpp", "fp8_adamw_expand_cuda_kernel.cu"]
    sources = [os.path.join(src, n) for n in names]
    if not all(os.path.exists(s) for s in sources):
        return None
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load
    # same nvcc options as the reference's setup.py (-O3, C++17, no fast-math)
    load(name="qoptim_cuda", sources=sources, build_directory=OUT,
         extra_cuda_cflags=["-O3", "-std=c++17",
                            "-gencode", "arch=compute_100a,code=sm_100a"],
         extra_cflags=["-O3", "-std=c++17"],
         is_python_module=False, verbose=verbose)
    so = os.path.join(OUT, "qoptim_cuda.so")
    return so if os.path.exists(so) else None


if __name__ == "__main__":
    arg = sys.argv[1] if len(sys.argv) > 1 else None
    print(stage_python(arg))
    if not os.path.exists(os.path.join(OUT, "qoptim_cuda.so")):
        print(build(arg, verbose=True))
