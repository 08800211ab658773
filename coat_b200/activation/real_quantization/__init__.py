"""Real (not simulated) FP8 quantization operators, the names the reference exports from
coat/activation/real_quantization/__init__.py:3-25."""
from ._dequantize import fp8_dequantize  # noqa: F401
from ._division import fp8_division  # noqa: F401
from ._division_transpose import fp8_division_transpose  # noqa: F401
from ._quantize import fp8_quantize  # noqa: F401
from ._quantize_perblock import fp8_quantize_perblock  # noqa: F401
from ._quantize_perblock_transpose import fp8_quantize_perblock_transpose  # noqa: F401
from ._quantize_perblock_transpose_pergroup import fp8_quantize_perblock_transpose_pergroup  # noqa: F401
from ._quantize_pertensor import fp8_quantize_pertensor  # noqa: F401
from ._quantize_pertensor_transpose import fp8_quantize_pertensor_transpose  # noqa: F401
from ._transpose import fp8_transpose  # noqa: F401
from .add_bwd import fp8_add_Ifp_Ifp_Ofp_Opt  # noqa: F401
from .add_fwd import fp8_add_Ifp_Ifp_Ofp_Og16  # noqa: F401
from .func_layernorm_noparam import fp8_layernorm_noparam_backward, fp8_layernorm_noparam_forward  # noqa: F401
from .func_layernorm_param import fp8_layernorm_param_backward, fp8_layernorm_param_forward  # noqa: F401
from .func_rmsnorm import fp8_rmsnorm_backward, fp8_rmsnorm_forward  # noqa: F401
from .gelu_bwd import fp8_gelu_backward  # noqa: F401
from .gelu_fwd import fp8_gelu_forward  # noqa: F401
from .mul_bwd import fp8_mul_backward  # noqa: F401
from .mul_fwd import fp8_mul_forward  # noqa: F401
from .silu_bwd import fp8_silu_backward  # noqa: F401
from .silu_fwd import fp8_silu_forward  # noqa: F401
from .linear import fp8_linear_backward, fp8_linear_forward  # noqa: F401
from ._quantize_transpose import fp8_quantize_transpose  # noqa: F401
from ._fused import fp8_mul_silu_backward, fp8_mul_silu_backward_joint, fp8_silu_mul_forward  # noqa: F401  (extensions: the gated product's two operators in one kernel, forward and backward)
