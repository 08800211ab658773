from ._ops import fp8_quantize_perblock_transpose  # noqa: F401
