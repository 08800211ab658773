"""The COAT Llama model around the decoder layers: embedding -> FP8 activation stream through the layers
-> final norm (-> LM head and loss).

Same class names, attribute names (hence state-dict keys) and data flow as coat/models/coat_llama.py:1206-1449
of the reference: `CoatLlamaModel` embeds the tokens, `Coat_quantize_bgn` opens the (bf16, FP8 codes, scales)
stream, every `CoatLlamaDecoderLayer` passes the triple on, `Coat_quantize_end` closes it (and opens the FP8
gradient stream in backward), then the final RMSNorm; `CoatLlamaForCausalLM` adds `lm_head` and the shifted
cross-entropy loss; `make_state_dict_compatible` renames the keys of a stock Llama checkpoint
(`self_attn.q_proj` -> `BeforeAttention.q_proj` and so on) so that it loads into these modules.

The classes are plain `nn.Module`s (no `PreTrainedModel` base, no generation or KV-cache plumbing: this is the
training model), so they do not depend on a particular transformers release.  The rotary tables are computed
once per forward and shared by all layers.  The loss is the token-mean cross entropy of the shifted logits,
computed in chunks of rows so that the fp32 logits of the whole batch never exist at once, each chunk through the
cross-entropy kernel that writes the gradient in place of the logits (the reference
delegates this to a fused linear-cross-entropy from Liger, coat_llama.py:1407-1411; it is not part of the FP8
path).
"""
from fnmatch import fnmatch
from typing import NamedTuple, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..activation.liger.cross_entropy import LigerCrossEntropyFunction

from ..activation.real_quantization.func_quantize import Coat_quantize_bgn, Coat_quantize_end
from ..utils._fp8_quantization_config import QuantizationConfig
from .coat_llama import CoatLlamaDecoderLayer, LlamaRMSNorm, llama_rotary_embeddings


class BaseModelOutput(NamedTuple):
    last_hidden_state: torch.Tensor


class CausalLMOutput(NamedTuple):
    loss: Optional[torch.Tensor]
    logits: Optional[torch.Tensor]


class CoatLlamaModel(nn.Module):
    """coat_llama.py:1206-1374: `embed_tokens`, `layers`, `norm` and the two stream modules."""

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.padding_idx = getattr(config, "pad_token_id", None)
        self.vocab_size = config.vocab_size
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size, self.padding_idx)
        self.layers = nn.ModuleList(CoatLlamaDecoderLayer(config, i) for i in range(config.num_hidden_layers))
        self.norm = LlamaRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.qargs = QuantizationConfig(**config.coat_fp8_args)
        self.quantize_input_before_block = Coat_quantize_bgn(self.qargs)
        self.quantize_output_after_block = Coat_quantize_end(self.qargs)
        self.apply(self._init_weights)

    def _init_weights(self, module):
        std = getattr(self.config, "initializer_range", 0.02)   # coat_llama.py:1195-1204
        if isinstance(module, nn.Linear):
            module.weight.data.normal_(mean=0.0, std=std)
            if module.bias is not None:
                module.bias.data.zero_()
        elif isinstance(module, nn.Embedding):
            module.weight.data.normal_(mean=0.0, std=std)
            if module.padding_idx is not None:
                module.weight.data[module.padding_idx].zero_()

    def get_input_embeddings(self):
        return self.embed_tokens

    def set_input_embeddings(self, value):
        self.embed_tokens = value

    def forward(self, input_ids: Optional[torch.LongTensor] = None, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.LongTensor] = None, inputs_embeds: Optional[torch.Tensor] = None,
                **kwargs):
        if (input_ids is None) == (inputs_embeds is None):
            raise ValueError("You must specify exactly one of input_ids or inputs_embeds")
        if inputs_embeds is None:
            inputs_embeds = self.embed_tokens(input_ids)
        bsz, q_len, _ = inputs_embeds.shape
        if position_ids is None:
            position_ids = torch.arange(q_len, device=inputs_embeds.device)[None, :]
        head_dim = getattr(self.config, "head_dim", None) or self.config.hidden_size // self.config.num_attention_heads
        position_embeddings = llama_rotary_embeddings(position_ids, head_dim, getattr(self.config, "rope_theta", 10000.0),
                                                      inputs_embeds.dtype)
        mask = self._attention_mask(attention_mask, bsz, q_len, inputs_embeds)
        hidden, q_hidden, s_hidden = self.quantize_input_before_block(inputs_embeds)
        for layer in self.layers:
            (hidden, q_hidden, s_hidden), = layer(hidden, q_hidden, s_hidden, attention_mask=mask,
                                                  position_ids=position_ids, position_embeddings=position_embeddings)
        hidden = self.quantize_output_after_block(hidden, q_hidden, s_hidden)
        return BaseModelOutput(self.norm(hidden))

    @staticmethod
    def _attention_mask(attention_mask, bsz, q_len, like):
        """None (pure causal attention, the fast path) unless the 2-D padding mask really masks something; then
        the additive [batch, 1, q, k] mask of causal AND not-padded."""
        if attention_mask is None or bool(attention_mask.all()):
            return None
        keep = torch.ones(q_len, q_len, dtype=torch.bool, device=like.device).tril()[None, None]
        keep = keep & attention_mask.to(torch.bool)[:, None, None, :]
        return torch.zeros(bsz, 1, q_len, q_len, dtype=like.dtype, device=like.device).masked_fill(~keep, float("-inf"))


def chunked_causal_lm_loss(hidden, lm_head_weight, labels, ignore_index=-100, chunk_rows=4096):
    """Mean cross entropy of position t predicting label t+1, with the logits of `chunk_rows` positions in
    fp32 at a time."""
    h = hidden[:, :-1, :].reshape(-1, hidden.shape[-1])
    y = labels[:, 1:].reshape(-1)
    n_valid = (y != ignore_index).sum().clamp(min=1)
    total = hidden.new_zeros((), dtype=torch.float32)
    for i in range(0, h.shape[0], chunk_rows):
        logits = F.linear(h[i:i + chunk_rows], lm_head_weight).float()
        if logits.is_cuda:
            # the loss head of the reference (LigerForCausalLMLoss): the gradient overwrites the chunk's logits, so
            # autograd keeps no second [rows, vocabulary] tensor (log-softmax) per chunk
            part, _ = LigerCrossEntropyFunction.apply(logits, y[i:i + chunk_rows], ignore_index, 0.0, 0.0, "sum")
        else:   # evaluation on the host (tests of the model's plumbing)
            part = F.cross_entropy(logits, y[i:i + chunk_rows], ignore_index=ignore_index, reduction="sum")
        total = total + part
    return total / n_valid


class CoatLlamaForCausalLM(nn.Module):
    """coat_llama.py:1377-1415: `model` + `lm_head` (bf16 linear; the head is not quantised in the reference
    either)."""
    _tied_weights_keys = ["lm_head.weight"]

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.model = CoatLlamaModel(config)
        self.vocab_size = config.vocab_size
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.lm_head.weight.data.normal_(mean=0.0, std=getattr(config, "initializer_range", 0.02))
        if getattr(config, "tie_word_embeddings", False):
            self.lm_head.weight = self.model.embed_tokens.weight

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
        hidden = self.model(input_ids=input_ids, attention_mask=attention_mask, position_ids=position_ids,
                            inputs_embeds=inputs_embeds).last_hidden_state
        loss = None
        if labels is not None:
            loss = chunked_causal_lm_loss(hidden, self.lm_head.weight, labels)
        want_logits = (labels is None) if return_logits is None else return_logits
        return CausalLMOutput(loss, self.lm_head(hidden) if want_logits else None)


_RENAMES = (
    ("self_attn.q_proj", "BeforeAttention.q_proj"),
    ("self_attn.k_proj", "BeforeAttention.k_proj"),
    ("self_attn.v_proj", "BeforeAttention.v_proj"),
    ("self_attn.o_proj", "AfterAttention.o_proj"),
    ("mlp.gate_proj", "MLPResidual.gate_proj"),
    ("mlp.up_proj", "MLPResidual.up_proj"),
    ("mlp.down_proj", "MLPResidual.down_proj"),
)


def make_state_dict_compatible(state_dict):
    """Keys of a stock Llama checkpoint renamed to this model's module names (coat_llama.py:1424-1449); keys
    that already carry the new names, and all others, pass unchanged."""
    out = {}
    for key, value in state_dict.items():
        for old, new in _RENAMES:
            if fnmatch(key, f"*{old}*"):
                key = key.replace(old, new)
                break
        out[key] = value
    return out
