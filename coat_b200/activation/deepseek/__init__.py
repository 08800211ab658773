from .fp8linear import FP8DeepSeekLinear  # noqa: F401
from .linear import fp8_deepseek_linear_backward, fp8_deepseek_linear_forward, gemm_fp8_fp8_bf16_nt  # noqa: F401
