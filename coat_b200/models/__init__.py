from .coat_llama import (  # noqa: F401
    CoatLlamaAfterAttentionResidual,
    CoatLlamaBeforeAttentionResidual,
    CoatLlamaConfig,
    CoatLlamaDecoderLayer,
    CoatLlamaMLPResidual,
    LlamaSdpaAttentionWithoutLinear,
)
from .coat_llama_model import (  # noqa: F401
    CoatLlamaForCausalLM,
    CoatLlamaModel,
    chunked_causal_lm_loss,
    make_state_dict_compatible,
)
from .coat_olmo import (  # noqa: F401
    CoatOLMo,
    CoatOLMoAfterAttentionResidual,
    CoatOLMoBeforeAttentionResidual,
    CoatOLMoBlock,
    CoatOLMoConfig,
    CoatOLMoMLPResidual,
    CoatOLMoSequentialBlock,
)
