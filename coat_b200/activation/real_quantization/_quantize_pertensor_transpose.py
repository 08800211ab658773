"""fp8_quantize_pertensor_transpose under the module path the reference uses (coat/activation/real_quantization/_quantize_pertensor_transpose.py)."""
from ._ops import fp8_quantize_pertensor_transpose  # noqa: F401
