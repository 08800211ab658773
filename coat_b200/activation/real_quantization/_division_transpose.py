"""fp8_division_transpose under the module path the reference uses (coat/activation/real_quantization/_division_transpose.py)."""
from ._ops import fp8_division_transpose  # noqa: F401
