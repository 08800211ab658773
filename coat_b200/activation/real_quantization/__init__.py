"""Real (not simulated) FP8 quantization operators, the names the reference exports from
coat/activation/real_quantization/__init__.py:3-25."""
from ._dequantize import fp8_dequantize  # noqa: F401
from ._division import fp8_division  # noqa: F401
from ._division_transpose import fp8_division_transpose  # noqa: F401
from ._quantize import fp8_quantize  # noqa: F401
from ._quantize_pertensor import fp8_quantize_pertensor  # noqa: F401
from ._quantize_pertensor_transpose import fp8_quantize_pertensor_transpose  # noqa: F401
from ._transpose import fp8_transpose  # noqa: F401
