"""fp8_rmsnorm_forward, fp8_rmsnorm_backward under the module path the reference uses (coat/activation/real_quantization/func_rmsnorm.py)."""
from ._fused import fp8_rmsnorm_forward, fp8_rmsnorm_backward  # noqa: F401
