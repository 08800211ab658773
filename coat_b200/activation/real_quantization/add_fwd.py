"""fp8_add_Ifp_Ifp_Ofp_Og16 under the module path the reference uses (coat/activation/real_quantization/add_fwd.py)."""
from ._fused import fp8_add_Ifp_Ifp_Ofp_Og16  # noqa: F401
