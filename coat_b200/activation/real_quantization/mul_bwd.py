"""fp8_mul_backward under the module path the reference uses (coat/activation/real_quantization/mul_bwd.py)."""
from ._fused import fp8_mul_backward  # noqa: F401
