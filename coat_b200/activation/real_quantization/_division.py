"""fp8_division under the module path the reference uses (coat/activation/real_quantization/_division.py)."""
from ._ops import fp8_division  # noqa: F401
