from ._ops import fp8_quantize_perblock  # noqa: F401
