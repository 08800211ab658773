"""fp8_silu_forward under the module path the reference uses (coat/activation/real_quantization/silu_fwd.py)."""
from ._fused import fp8_silu_forward  # noqa: F401
