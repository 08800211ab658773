"""fp8_quantize under the module path the reference uses (coat/activation/real_quantization/_quantize.py)."""
from ._ops import fp8_quantize  # noqa: F401
