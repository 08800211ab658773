"""fp8_add_Ifp_Ifp_Ofp_Opt under the module path the reference uses (coat/activation/real_quantization/add_bwd.py)."""
from ._fused import fp8_add_Ifp_Ifp_Ofp_Opt  # noqa: F401
