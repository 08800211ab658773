"""fp8_mul_forward under the module path the reference uses (coat/activation/real_quantization/mul_fwd.py)."""
from ._fused import fp8_mul_forward  # noqa: F401
