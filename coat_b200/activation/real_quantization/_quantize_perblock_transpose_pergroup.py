from ._ops import fp8_quantize_perblock_transpose_pergroup  # noqa: F401
