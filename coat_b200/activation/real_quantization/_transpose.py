"""fp8_transpose under the module path the reference uses (coat/activation/real_quantization/_transpose.py)."""
from ._ops import fp8_transpose  # noqa: F401
