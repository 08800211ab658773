"""fp8_quantize_pertensor under the module path the reference uses (coat/activation/real_quantization/_quantize_pertensor.py)."""
from ._ops import fp8_quantize_pertensor  # noqa: F401
