from ._fp8_quantization_config import QuantizationConfig  # noqa: F401
