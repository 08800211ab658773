"""fp8_gelu_forward under the module path the reference uses (coat/activation/real_quantization/gelu_fwd.py)."""
from ._fused import fp8_gelu_forward  # noqa: F401
