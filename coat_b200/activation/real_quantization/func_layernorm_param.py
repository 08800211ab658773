"""fp8_layernorm_param_forward, fp8_layernorm_param_backward under the module path the reference uses (coat/activation/real_quantization/func_layernorm_param.py)."""
from ._fused import fp8_layernorm_param_backward, fp8_layernorm_param_forward  # noqa: F401
