"""fp8_silu_backward under the module path the reference uses (coat/activation/real_quantization/silu_bwd.py)."""
from ._fused import fp8_silu_backward  # noqa: F401
