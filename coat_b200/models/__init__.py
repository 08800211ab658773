from .coat_llama import (  # noqa: F401
    CoatLlamaAfterAttentionResidual,
    CoatLlamaBeforeAttentionResidual,
    CoatLlamaConfig,
    CoatLlamaDecoderLayer,
    CoatLlamaMLPResidual,
    LlamaSdpaAttentionWithoutLinear,
)
