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
