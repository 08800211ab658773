"""Test-side access to the checkers: the C restatement (oracle/adamw.py) and, when it
has been built, the reference's own CUDA extension compiled by oracle/build_ref.py."""
import importlib
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def load_ref_qoptim():
    """The reference's `qoptim_cuda` module built into oracle/_ref, or None."""
    so = os.path.join(REF_DIR, "qoptim_cuda.so")
    if not os.path.exists(so):
        return None
    import torch  # noqa: F401  (the extension links against torch)
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        return importlib.import_module("qoptim_cuda")
    except Exception:
        return None


_REF_TRITON = None


def _one_config(obj, seen):
    """Walk a Triton kernel wrapper chain (Heuristics -> Autotuner -> JITFunction) and keep ONE of the
    autotuner's own candidate configurations, so that nothing is benchmarked: every candidate computes
    the same values (the kernels reduce with max only, tile by tile), the choice only affects speed.
    The smallest tile of the list is kept (least register pressure, quickest to compile)."""
    from triton.runtime.autotuner import Autotuner
    while obj is not None and id(obj) not in seen:
        seen.add(id(obj))
        if isinstance(obj, Autotuner) and len(obj.configs) > 1:
            def area(c):
                kw = c.kwargs
                return kw.get("BLOCK_M", 1) * kw.get("BLOCK_N", 1), c.num_warps, c.num_stages
            obj.configs = [min(obj.configs, key=area)]
        obj = getattr(obj, "fn", None)


def load_ref_triton():
    """The reference's operator layer (its Triton kernels and python wrappers) as staged by
    oracle/build_ref.py into oracle/_ref/coat_ref/, or None when it has not been staged.  GPU only."""
    global _REF_TRITON
    if _REF_TRITON is not None:
        return _REF_TRITON
    pkg = os.path.join(REF_DIR, "coat_ref", "activation", "real_quantization")
    if not os.path.isdir(pkg):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    mod = importlib.import_module("coat_ref.activation.real_quantization")
    seen = set()
    for name in sorted(os.listdir(pkg)):
        if not name.endswith(".py") or name == "__init__.py":
            continue
        try:
            sub = importlib.import_module(f"coat_ref.activation.real_quantization.{name[:-3]}")
        except Exception:
            continue
        for val in list(vars(sub).values()):
            for k in (val.values() if isinstance(val, dict) else (val,)):
                if hasattr(k, "fn"):
                    _one_config(k, seen)
    _REF_TRITON = mod
    return mod


def ref_module(name):
    """A submodule of the staged reference package, e.g. ref_module('_quantize_transpose')."""
    load_ref_triton()
    return importlib.import_module(f"coat_ref.activation.real_quantization.{name}")
