"""fp8_dequantize under the module path the reference uses (coat/activation/real_quantization/_dequantize.py)."""
from ._ops import fp8_dequantize  # noqa: F401
