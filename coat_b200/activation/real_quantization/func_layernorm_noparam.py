"""fp8_layernorm_noparam_forward, fp8_layernorm_noparam_backward under the module path the reference uses (coat/activation/real_quantization/func_layernorm_noparam.py)."""
from ._fused import fp8_layernorm_noparam_backward, fp8_layernorm_noparam_forward  # noqa: F401
