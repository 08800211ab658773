"""fp8_quantize_transpose under the module path the reference uses (coat/activation/real_quantization/_quantize_transpose.py)."""
from ._ops import fp8_quantize_transpose  # noqa: F401
