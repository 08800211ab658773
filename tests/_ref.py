"""Test-side access to the checkers staged by oracle/build_ref.py: the reference's compiled optimizer extension and
its Triton operator layer (oracle/ref_loader.py holds the loaders)."""
from oracle.ref_loader import REF_DIR, load_ref_qoptim, load_ref_triton, ref_module  # noqa: F401
from oracle.ref_loader import load_ref_optimizer  # noqa: F401,E402
