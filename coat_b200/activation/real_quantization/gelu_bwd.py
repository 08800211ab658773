"""fp8_gelu_backward under the module path the reference uses (coat/activation/real_quantization/gelu_bwd.py)."""
from ._fused import fp8_gelu_backward  # noqa: F401
