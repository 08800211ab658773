"""The transformers-facing form of the COAT Llama model: `CoatLlamaConfig` (a `LlamaConfig` with `model_type =
"fp8_llama"` and the `coat_fp8_args` dictionary), `CoatLlamaPreTrainedModel`, `CoatLlamaModel` and
`CoatLlamaForCausalLM` as `PreTrainedModel`s registered with `AutoConfig` / `AutoModel` / `AutoModelForCausalLM`
(coat/models/coat_llama.py:106-107, 1183-1421 of the reference), and the checkpoint converter
`download_and_convert_llama` (coat/models/coat_llama_convert_from_hf.py:20-62).

Only `save_pretrained` / `from_pretrained` / `from_config`, weight initialisation and the output classes come from
transformers; modules, state-dict keys and the forward passes are those of coat_llama_model.py (the classes here
build the same attributes and borrow its forward functions), so a checkpoint written by the reference's classes
loads here and the other way round.  Importing this module needs transformers; nothing else in the package does.
"""
import os
from dataclasses import asdict, dataclass, field

import torch.nn as nn
from transformers import AutoConfig, AutoModel, AutoModelForCausalLM, LlamaConfig, PreTrainedModel
from transformers.modeling_outputs import BaseModelOutputWithPast, CausalLMOutputWithPast

try:
    import transformers.initialization  # noqa: F401
    _HAS_FLAGGED_INIT = True
except ImportError:
    _HAS_FLAGGED_INIT = False

from ..activation.real_quantization.func_quantize import Coat_quantize_bgn, Coat_quantize_end
from ..utils._fp8_quantization_config import QuantizationConfig
from . import coat_llama_model as plain
from .coat_llama import CoatLlamaDecoderLayer, LlamaRMSNorm


class CoatLlamaConfig(LlamaConfig):
    model_type = "fp8_llama"

    def __init__(self, coat_fp8_args=None, **kwargs):
        super().__init__(**kwargs)
        self.coat_fp8_args = dict(coat_fp8_args or {})


class CoatLlamaPreTrainedModel(PreTrainedModel):
    config_class = CoatLlamaConfig
    base_model_prefix = "model"
    supports_gradient_checkpointing = False
    _no_split_modules = ["CoatLlamaDecoderLayer"]
    _supports_sdpa = True

    def _init_weights(self, module):
        # coat_llama.py:1195-1204.  Current transformers releases initialise Linear / Embedding / *RMSNorm modules this
        # way in the base class, through functions that leave weights already loaded from a checkpoint alone; the
        # explicit form is for releases that expect every model to bring its own.
        if _HAS_FLAGGED_INIT:
            return super()._init_weights(module)
        std = self.config.initializer_range
        if isinstance(module, nn.Linear):
            module.weight.data.normal_(mean=0.0, std=std)
            if module.bias is not None:
                module.bias.data.zero_()
        elif isinstance(module, nn.Embedding):
            module.weight.data.normal_(mean=0.0, std=std)
            if module.padding_idx is not None:
                module.weight.data[module.padding_idx].zero_()
        elif isinstance(module, LlamaRMSNorm):
            module.weight.data.fill_(1.0)


class CoatLlamaModel(CoatLlamaPreTrainedModel):
    """coat_llama.py:1206-1374."""

    def __init__(self, config: CoatLlamaConfig):
        super().__init__(config)
        self.padding_idx = config.pad_token_id
        self.vocab_size = config.vocab_size
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size, self.padding_idx)
        self.layers = nn.ModuleList(CoatLlamaDecoderLayer(config, i) for i in range(config.num_hidden_layers))
        self.norm = LlamaRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.qargs = QuantizationConfig(**config.coat_fp8_args)
        self.quantize_input_before_block = Coat_quantize_bgn(self.qargs)
        self.quantize_output_after_block = Coat_quantize_end(self.qargs)
        self.post_init()

    def get_input_embeddings(self):
        return self.embed_tokens

    def set_input_embeddings(self, value):
        self.embed_tokens = value

    _attention_mask = staticmethod(plain.CoatLlamaModel._attention_mask)

    def forward(self, input_ids=None, attention_mask=None, position_ids=None, inputs_embeds=None, **kwargs):
        out = plain.CoatLlamaModel.forward(self, input_ids=input_ids, attention_mask=attention_mask,
                                           position_ids=position_ids, inputs_embeds=inputs_embeds)
        return BaseModelOutputWithPast(last_hidden_state=out.last_hidden_state)


class CoatLlamaForCausalLM(CoatLlamaPreTrainedModel):
    """coat_llama.py:1377-1415."""
    _tied_weights_keys = {"lm_head.weight": "model.embed_tokens.weight"}

    def __init__(self, config: CoatLlamaConfig):
        super().__init__(config)
        self.model = CoatLlamaModel(config)
        self.vocab_size = config.vocab_size
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.post_init()

    def get_input_embeddings(self):
        return self.model.embed_tokens

    def set_input_embeddings(self, value):
        self.model.embed_tokens = value

    def get_output_embeddings(self):
        return self.lm_head

    def set_output_embeddings(self, new_embeddings):
        self.lm_head = new_embeddings

    def set_decoder(self, decoder):
        self.model = decoder

    def get_decoder(self):
        return self.model

    def forward(self, input_ids=None, attention_mask=None, position_ids=None, inputs_embeds=None, labels=None,
                return_logits=None, **kwargs):
        out = plain.CoatLlamaForCausalLM.forward(self, input_ids=input_ids, attention_mask=attention_mask,
                                                 position_ids=position_ids, inputs_embeds=inputs_embeds, labels=labels,
                                                 return_logits=return_logits)
        return CausalLMOutputWithPast(loss=out.loss, logits=out.logits)


AutoConfig.register("fp8_llama", CoatLlamaConfig)
AutoModel.register(CoatLlamaConfig, CoatLlamaModel)
AutoModelForCausalLM.register(CoatLlamaConfig, CoatLlamaForCausalLM)


@dataclass
class ConvertArguments:
    model_name: str = field(metadata={"help": "The model name or path of the stock Llama model"})
    save_path: str = field(metadata={"help": "The path where the converted model weights will be saved"})
    cache_dir: str = field(default=None, metadata={"help": "Directory to cache the model"})


def download_and_convert_llama(convert_args: ConvertArguments, quantization_args: QuantizationConfig):
    """Load a stock Llama checkpoint (a local directory, or a hub name where there is a network), rename its keys with
    `make_state_dict_compatible`, load them into a `CoatLlamaForCausalLM` whose configuration carries the quantization
    arguments, and `save_pretrained` it."""
    model = AutoModelForCausalLM.from_pretrained(convert_args.model_name, cache_dir=convert_args.cache_dir)
    config = AutoConfig.from_pretrained(convert_args.model_name, cache_dir=convert_args.cache_dir)
    compatible = plain.make_state_dict_compatible(model.state_dict())
    fields = config.to_dict()
    for k in ("model_type", "architectures", "transformers_version"):
        fields.pop(k, None)
    fp8_config = CoatLlamaConfig(**fields)
    fp8_config.coat_fp8_args = asdict(quantization_args)
    converted = AutoModelForCausalLM.from_config(fp8_config)
    converted.load_state_dict(compatible)
    os.makedirs(convert_args.save_path, exist_ok=True)
    converted.save_pretrained(convert_args.save_path)
    return converted


if __name__ == "__main__":
    import transformers
    parser = transformers.HfArgumentParser((ConvertArguments, QuantizationConfig))
    download_and_convert_llama(*parser.parse_args_into_dataclasses())
