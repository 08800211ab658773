"""The COAT OLMo transformer block on the B200 operators.

Same class names, constructor arguments, forward signatures and data flow as coat/models/coat_olmo.py of the
reference (the block its per-layer benchmark, benchmark/benchmark_olmolayer.py, times): a sequential block is
three autograd blocks that pass the triple (bf16 hidden states, their 1x16 FP8 codes, the group scales) on,

    BeforeAttentionResidual (:94-244)   LayerNorm without parameters on the FP8 input -> per-tensor FP8 ->
                                        ONE fused q/k/v projection (`att_proj`)
    attention (:769-888)                RoPE in full precision + causal attention on bf16 q/k/v (torch SDPA)
    AfterAttentionResidual  (:247-380)  per-tensor FP8 of the attention output -> `attn_out` -> residual add
                                        fused with the 1x16 quantisation of the sum
    MLPResidual             (:383-645)  LayerNorm -> `ff_proj` (up and gate halves, in that order) with the
                                        1x16-quantising epilogue -> SiLU(gate) * up -> `ff_out` -> residual add

and whose backward passes run the mirrored chain on E5M2 gradients; in the MLP the gradients towards the up and
the gate halves share ONE per-tensor scale (the reference concatenates them before it quantises, :603-611).
What differs from the Llama layer: the norm (LayerNorm, no weight, no bias), the fused projections, and OLMo's
rotary embedding computed in fp32.  `CoatOLMoConfig` is a plain attribute bag with the fields of the host
trainer's ModelConfig that the block reads (any object with those attributes works).  `CoatOLMo` at the end of the
file is the model around the blocks (embedding, the FP8 stream through the blocks, final norm, output projection) with
the reference's module names; the trainer, its yaml configuration, checkpointing and FSDP wrapping policies stay with
the host framework.

Two things are done differently from the reference's composition without changing a bit of the result:
the up and gate halves of `ff_proj` come from two GEMMs over the two halves of the weight codes (the halves
of one fused result would be strided views, which every following operator would first have to copy), and
the gated product and its backward run in one kernel each.
"""
import math
from typing import NamedTuple, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..activation.real_quantization.func_quantize import Coat_quantize_bgn, Coat_quantize_end
from ..activation.real_quantization import (
    fp8_add_Ifp_Ifp_Ofp_Og16,
    fp8_add_Ifp_Ifp_Ofp_Opt,
    fp8_division_transpose,
    fp8_layernorm_noparam_backward,
    fp8_layernorm_noparam_forward,
    fp8_linear_backward,
    fp8_linear_forward,
    fp8_mul_silu_backward_joint,
    fp8_quantize_pertensor,
    fp8_quantize_pertensor_transpose,
    fp8_silu_mul_forward,
    fp8_transpose,
)
from ..utils._fp8_quantization_config import QuantizationConfig
from ..utils._fp8_weightcache import FP8CacheWeightModule
from ..utils._fp8manager import FP8Manager
from .coat_llama import _as_e4m3, _backward_weight_t, _forward_weights, _FusedRotary, _fwobits, _rotate_half


class CoatOLMoConfig:
    """The fields of OLMo's ModelConfig (examples/OLMo/olmo/config.py of the reference's vendored trainer) that the
    block reads, with OLMo-7B's values as defaults (examples/OLMo/configs/coat/OLMo-7B-COAT-Activation.yaml:9-36)."""

    def __init__(self, d_model=4096, n_heads=32, n_kv_heads=None, n_layers=32, mlp_ratio=4, mlp_hidden_size=22016,
                 activation_type="swiglu", include_bias=False, rope=True, rope_theta=10000.0, rope_full_precision=True,
                 clip_qkv=None, attention_dropout=0.0, residual_dropout=0.0, attention_layer_norm=False,
                 layer_norm_with_affine=False, layer_norm_eps=1e-5, max_sequence_length=2048, init_device=None,
                 init_std=0.02, norm_after=False, block_type="sequential", multi_query_attention=False, **kwargs):
        self.d_model, self.n_heads, self.n_kv_heads, self.n_layers = d_model, n_heads, n_kv_heads, n_layers
        self.mlp_ratio, self.mlp_hidden_size = mlp_ratio, mlp_hidden_size
        self.activation_type = activation_type
        self.include_bias = include_bias
        self.rope, self.rope_theta, self.rope_full_precision = rope, rope_theta, rope_full_precision
        self.clip_qkv = clip_qkv
        self.attention_dropout, self.residual_dropout = attention_dropout, residual_dropout
        self.attention_layer_norm = attention_layer_norm
        self.layer_norm_with_affine, self.layer_norm_eps = layer_norm_with_affine, layer_norm_eps
        self.max_sequence_length = max_sequence_length
        self.init_device, self.init_std = init_device, init_std
        self.norm_after, self.block_type = norm_after, block_type
        self.multi_query_attention = multi_query_attention
        for k, v in kwargs.items():
            setattr(self, k, v)

    @property
    def effective_n_kv_heads(self):
        if self.n_kv_heads is None:
            return 1 if self.multi_query_attention else self.n_heads
        return self.n_kv_heads


def _activation_name(config):
    return str(getattr(config.activation_type, "value", config.activation_type)).lower()


def _device(config):
    dev = getattr(config, "init_device", None)
    return None if dev in (None, "meta") else dev


def _check_supported(config):
    if _activation_name(config) != "swiglu":
        raise NotImplementedError("the quantised OLMo block is written for the swiglu activation, as the reference's "
                                  "(coat_olmo.py:518-526 splits ff_proj into up and gate whatever the configuration says)")
    if getattr(config, "layer_norm_with_affine", False):
        raise NotImplementedError("the quantised OLMo block applies a LayerNorm without parameters")
    if getattr(config, "include_bias", False):
        raise NotImplementedError("the FP8 linear layers of the block carry no bias (coat_olmo.py:199,326,520,531)")


def _plain_layernorm(x, eps=1e-5):
    return F.layer_norm(x, x.shape[-1:], None, None, eps)


def _prepared(module, names):
    """Arguments (origin, codes, transposed codes, scale) per weight for the autograd blocks."""
    args = []
    with torch.no_grad():
        for name in names:
            weight = getattr(module, name).weight
            prepared = module.prepare_weight(weight, name, FP8Manager.is_first_microbatch)
            if module.qargs.weight_memory_efficient:
                args += [weight, None, None, prepared]
            else:
                args += [weight, prepared[0], prepared[1], prepared[2]]
    return args


# =====================================================================================================
# Before attention: LayerNorm + the fused q/k/v projection
# =====================================================================================================
class _CoatOLMoBeforeAttentionResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, re_x, in_x, in_s, weight1_origin, weight1, weight1_t, weight1_s, group_size, fwobits, layer_id,
                config, qargs, eps=1e-5):
        if fwobits["fabit"] != "E4M3":
            raise ValueError("fabit should be E4M3")
        in_x = _as_e4m3(in_x)
        ln_x, ln_s, ln_x_t, ln_utils = fp8_layernorm_noparam_forward(in_x, in_s, group_size, eps,
                                                                     transpose_output_2d=True)
        (weight1,) = _forward_weights((weight1_origin,), (weight1,), (weight1_s,), qargs, fwobits["fwbit"])
        fc1_x = fp8_linear_forward(ln_x, ln_s, weight1, weight1_s, False, group_size)

        ctx.save_for_backward(in_x, in_s, ln_x_t, ln_s)
        if qargs.weight_memory_efficient:
            assert weight1_t is None
            ctx.weight = weight1_origin, weight1_s
        else:
            ctx.weight = weight1_t, weight1_s
        ctx.group_size = group_size
        ctx.ln_utils = ln_utils
        ctx.utils = fwobits, layer_id, config, qargs
        return re_x, fc1_x

    @staticmethod
    def backward(ctx, fp_grad, flash_g):
        in_x, in_s, ln_x_t, ln_s = ctx.saved_tensors
        saved_w, weight1_s = ctx.weight
        group_size = ctx.group_size
        mean, rstd, num_warps = ctx.ln_utils
        fwobits, layer_id, config, qargs = ctx.utils

        # the gradient of q, k and v in one tensor: dgrad wants it as it is, wgrad its transposed copy
        flash_g, flash_gs, flash_g_t = fp8_quantize_pertensor_transpose(flash_g, group_size, fwobits["babit"],
                                                                        transpose_output_2d=True, stochastic=False)
        weight1_t = _backward_weight_t(saved_w, weight1_s, qargs, fwobits["fwbit"])
        fc1_g, att_proj_wg = fp8_linear_backward(ln_x_t, ln_s, flash_g, flash_gs, flash_g_t, weight1_t, weight1_s,
                                                 group_size)
        in_g = fp8_layernorm_noparam_backward(in_x, in_s, fc1_g, group_size, mean, rstd, num_warps)
        re_g, (in_g, in_sg, in_sg_g16) = fp8_add_Ifp_Ifp_Ofp_Opt(fp_grad, in_g, group_size, fwobits["babit"],
                                                                 stochastic=False)
        # the group scales, not the tensor scale, go back: the shape must match the forward's scale input
        return re_g, _as_e4m3(in_g), in_sg_g16, att_proj_wg, None, None, None, None, None, None, None, None, None


class CoatOLMoBeforeAttentionResidual(FP8CacheWeightModule):
    """Residual pass-through, LayerNorm and the fused q/k/v projection."""

    def __init__(self, config, qargs: QuantizationConfig, layer_id, fused_dims: tuple):
        super().__init__(config, qargs, layer_id)
        self.qargs = qargs
        self.fwobits = _fwobits(qargs)
        self.ln_normalized_shape = config.d_model
        self.att_proj = nn.Linear(config.d_model, sum(fused_dims), bias=config.include_bias, device=_device(config))

    def forward(self, re_x, x, s):
        if not self.training:
            return re_x, self.att_proj(_plain_layernorm(re_x))
        return _CoatOLMoBeforeAttentionResidual.apply(re_x, x, s, *_prepared(self, ("att_proj",)),
                                                      self.qargs.group_size, self.fwobits, self.layer_id, self.config,
                                                      self.qargs)


# =====================================================================================================
# After attention: output projection + residual
# =====================================================================================================
class _CoatOLMoAfterAttentionResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, re_x, flash_x, weight2_origin, weight2, weight2_t, weight2_s, group_size, fwobits, layer_id,
                config, qargs):
        flash_qx, flash_s, _ = fp8_quantize_pertensor(flash_x, group_size, fwobits["fabit"])
        (weight2,) = _forward_weights((weight2_origin,), (weight2,), (weight2_s,), qargs, fwobits["fwbit"])
        fc2_x = fp8_linear_forward(flash_qx, flash_s, weight2, weight2_s, False, group_size)
        fp_x, (out_x, out_s) = fp8_add_Ifp_Ifp_Ofp_Og16(re_x, fc2_x, flash_qx.dtype, group_size)

        # the bf16 attention output is kept (not its FP8 copy): backward re-derives the transposed codes
        ctx.save_for_backward(flash_x, flash_s)
        if qargs.weight_memory_efficient:
            assert weight2_t is None
            ctx.weight = weight2_origin, weight2_s
        else:
            ctx.weight = weight2_t, weight2_s
        ctx.group_size = group_size
        ctx.utils = fwobits, layer_id, config, qargs
        return fp_x, _as_e4m3(out_x), out_s

    @staticmethod
    def backward(ctx, fp_grad, out_g, out_gs):
        flash_x, flash_s = ctx.saved_tensors
        saved_w, weight2_s = ctx.weight
        group_size = ctx.group_size
        fwobits, layer_id, config, qargs = ctx.utils
        if fwobits["babit"] != "E5M2":
            raise ValueError("babit should be E5M2")
        out_g = out_g.view(torch.float8_e5m2)
        out_gs_max = out_gs.max()

        out_g_t = fp8_transpose(out_g, transpose_output_2d=True)
        flash_x_t, flash_s = fp8_division_transpose(flash_x, group_size, fwobits["fabit"], flash_s, stochastic=False,
                                                    only_transposed=True)
        weight2_t = _backward_weight_t(saved_w, weight2_s, qargs, fwobits["fwbit"])
        fc2_g, attn_out_wg = fp8_linear_backward(flash_x_t, flash_s, out_g, out_gs_max, out_g_t, weight2_t, weight2_s,
                                                 group_size)
        return fp_grad, fc2_g, attn_out_wg, None, None, None, None, None, None, None, None


class CoatOLMoAfterAttentionResidual(FP8CacheWeightModule):
    """The attention output projection and the residual add."""

    def __init__(self, config, qargs: QuantizationConfig, layer_id):
        super().__init__(config, qargs, layer_id)
        self.qargs = qargs
        self.fwobits = _fwobits(qargs)
        self.attn_out = nn.Linear(config.d_model, config.d_model, bias=config.include_bias, device=_device(config))

    def forward(self, re_x, in_x):
        if not self.training:
            return re_x + self.attn_out(in_x), None, None
        return _CoatOLMoAfterAttentionResidual.apply(re_x, in_x, *_prepared(self, ("attn_out",)),
                                                     self.qargs.group_size, self.fwobits, self.layer_id, self.config,
                                                     self.qargs)


# =====================================================================================================
# MLP: LayerNorm + ff_proj (up | gate) + SiLU(gate) * up + ff_out + residual
# =====================================================================================================
class _CoatOLMoMLPResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, re_x, in_x, in_s, weight1_origin, weight1, weight1_t, weight1_s, weight2_origin, weight2,
                weight2_t, weight2_s, group_size, fwobits, layer_id, config, qargs, eps=1e-5):
        if fwobits["fabit"] != "E4M3":
            raise ValueError("fabit should be E4M3")
        in_x = _as_e4m3(in_x)
        ln_x, ln_s, ln_x_t, ln_utils = fp8_layernorm_noparam_forward(in_x, in_s, group_size, eps,
                                                                     transpose_output_2d=True)
        origins, scales = (weight1_origin, weight2_origin), (weight1_s, weight2_s)
        weight1, weight2 = _forward_weights(origins, (weight1, weight2), scales, qargs, fwobits["fwbit"])

        # ff_proj: rows [0, I) of the weight give `up`, rows [I, 2I) give `gate` (the order of the reference's
        # `fc1_x.chunk(2, dim=-1)`); each half leaves its GEMM already quantised in 1x16 groups
        half = weight1.shape[0] // 2
        up_x, up_s = fp8_linear_forward(ln_x, ln_s, weight1[:half], weight1_s, True, group_size)
        gate_x, gate_s = fp8_linear_forward(ln_x, ln_s, weight1[half:], weight1_s, True, group_size)
        # (one kernel for fp8_silu_forward followed by fp8_mul_forward: same bits)
        (silu_x, silu_s), (mul_x, mul_s, mul_x_t) = fp8_silu_mul_forward(gate_x, gate_s, up_x, up_s, group_size,
                                                                         transpose_output_2d=True)
        fc2_x = fp8_linear_forward(mul_x, mul_s, weight2, weight2_s, False, group_size)
        fp_x, (out_x, out_s) = fp8_add_Ifp_Ifp_Ofp_Og16(re_x, fc2_x, mul_x.dtype, group_size)

        ctx.save_for_backward(in_x, in_s, ln_x_t, ln_s, gate_x, gate_s, up_x, up_s, silu_x, silu_s, mul_x_t, mul_s)
        if qargs.weight_memory_efficient:
            assert weight1_t is None and weight2_t is None
            ctx.weight = origins, scales
        else:
            ctx.weight = (weight1_t, weight2_t), scales
        ctx.group_size = group_size
        ctx.ln_utils = ln_utils
        ctx.utils = fwobits, layer_id, config, qargs
        return fp_x, _as_e4m3(out_x), out_s

    @staticmethod
    def backward(ctx, fp_grad, out_g, out_gs):
        in_x, in_s, ln_x_t, ln_s, gate_x, gate_s, up_x, up_s, silu_x, silu_s, mul_x_t, mul_s = ctx.saved_tensors
        (saved_w1, saved_w2), (weight1_s, weight2_s) = ctx.weight
        group_size = ctx.group_size
        mean, rstd, num_warps = ctx.ln_utils
        fwobits, layer_id, config, qargs = ctx.utils
        if fwobits["babit"] != "E5M2":
            raise ValueError("babit should be E5M2")
        out_g = out_g.view(torch.float8_e5m2)
        out_gs_max = out_gs.max()

        # ff_out
        out_g_t = fp8_transpose(out_g, transpose_output_2d=True)
        weight2_t = _backward_weight_t(saved_w2, weight2_s, qargs, fwobits["fwbit"])
        fc2_g, weight2_grad = fp8_linear_backward(mul_x_t, mul_s, out_g, out_gs_max, out_g_t, weight2_t, weight2_s,
                                                  group_size)
        del out_g, out_g_t, weight2_t

        # Mul and SiLU backward, then `cat([d_up, d_gate], -1)` quantised with ONE per-tensor scale (the larger of
        # the two gradients' scales) together with its transposed copy: one elementwise kernel, two division
        # passes that write into the halves of the joint buffers
        gateup_g, gateup_gs, gateup_g_t = fp8_mul_silu_backward_joint(silu_x, silu_s, up_x, up_s, gate_x, gate_s,
                                                                      fc2_g, group_size, fwobits["babit"])
        weight1_t = _backward_weight_t(saved_w1, weight1_s, qargs, fwobits["fwbit"])
        fc1_g, weight1_grad = fp8_linear_backward(ln_x_t, ln_s, gateup_g, gateup_gs, gateup_g_t, weight1_t, weight1_s,
                                                  group_size)
        in_g = fp8_layernorm_noparam_backward(in_x, in_s, fc1_g, group_size, mean, rstd, num_warps)
        re_g, (in_g, in_sg, in_sg_g16) = fp8_add_Ifp_Ifp_Ofp_Opt(fp_grad, in_g, group_size, fwobits["babit"],
                                                                 stochastic=False)
        return (re_g, _as_e4m3(in_g), in_sg_g16, weight1_grad, None, None, None, weight2_grad, None, None, None,
                None, None, None, None, None, None)


class CoatOLMoMLPResidual(FP8CacheWeightModule):
    """Residual, LayerNorm and the gated MLP."""

    def __init__(self, config, qargs: QuantizationConfig, layer_id, hidden_size: int):
        super().__init__(config, qargs, layer_id)
        self.qargs = qargs
        self.fwobits = _fwobits(qargs)
        self.ln_normalized_shape = config.d_model
        self.act_output_multiplier = 0.5 if _activation_name(config) == "swiglu" else 1
        self.ff_proj = nn.Linear(config.d_model, hidden_size, bias=config.include_bias, device=_device(config))
        self.ff_out = nn.Linear(int(self.act_output_multiplier * hidden_size), config.d_model,
                                bias=config.include_bias, device=_device(config))

    def forward(self, re_x, x, s):
        if not self.training:
            up, gate = self.ff_proj(_plain_layernorm(re_x)).chunk(2, dim=-1)
            return re_x + self.ff_out(F.silu(gate) * up), None, None
        return _CoatOLMoMLPResidual.apply(re_x, x, s, *_prepared(self, ("ff_proj", "ff_out")), self.qargs.group_size,
                                          self.fwobits, self.layer_id, self.config, self.qargs)


# =====================================================================================================
# The block
# =====================================================================================================
def olmo_rotary_tables(seq_len, head_dim, rope_theta, device):
    """fp32 sin / cos of shape [1, seq_len, head_dim] (olmo/model.py:266-292 of the vendored trainer)."""
    inv_freq = 1.0 / (rope_theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float) / head_dim))
    seq = torch.arange(seq_len, device=device, dtype=torch.float)
    freqs = torch.outer(seq, inv_freq)
    positions = torch.cat((freqs, freqs), dim=-1)
    return positions.sin()[None].contiguous(), positions.cos()[None].contiguous()


class CoatOLMoBlock(nn.Module):
    """Base of the block implementations (coat_olmo.py:648-907): dimensions, rotary tables and attention."""

    def __init__(self, layer_id: int, config, qargs: QuantizationConfig, cache=None):
        super().__init__()
        self.layer_id = layer_id
        self.config = config
        self.qargs = qargs
        self.hidden_size = (config.mlp_hidden_size if config.mlp_hidden_size is not None
                            else config.mlp_ratio * config.d_model)
        self._cache = cache if cache is not None else {}
        assert config.d_model % config.n_heads == 0
        if getattr(config, "attention_layer_norm", False):
            raise NotImplementedError("q/k layer norms are not part of the quantised block")
        if config.clip_qkv is not None:
            assert config.clip_qkv > 0

    def _rotary(self, seq_len, device):
        sin, cos = self._cache.get("rope_pos_sin"), self._cache.get("rope_pos_cos")
        if sin is None or sin.shape[1] < seq_len or sin.device != device:
            sin, cos = olmo_rotary_tables(max(seq_len, getattr(self.config, "max_sequence_length", 0) or 0),
                                          self.config.d_model // self.config.n_heads,
                                          getattr(self.config, "rope_theta", 10000.0), device)
            self._cache["rope_pos_sin"], self._cache["rope_pos_cos"] = sin, cos
        return sin[:, :seq_len], cos[:, :seq_len]

    def attention(self, q, k, v, attention_bias=None, layer_past=None, use_cache=False, max_doc_len=None,
                  cu_doc_lens=None):
        """RoPE + scaled-dot-product attention on projected q/k/v [B, T, heads * head_dim] (views into the fused
        projection's output are fine); returns ([B, T, d_model], None)."""
        if layer_past is not None or use_cache:
            raise NotImplementedError("the training block keeps no KV cache")
        if max_doc_len is not None or cu_doc_lens is not None:
            raise NotImplementedError("document masking needs the host trainer's variable-length attention")
        B, T, C = q.size()
        cfg = self.config
        hd = C // cfg.n_heads
        n_kv = cfg.effective_n_kv_heads
        q = q.view(B, T, cfg.n_heads, hd)
        k = k.view(B, T, n_kv, hd)
        v = v.view(B, T, n_kv, hd).transpose(1, 2)
        if cfg.rope:
            sin, cos = self._rotary(T, q.device)
            full = getattr(cfg, "rope_full_precision", True)
            if not full:
                sin, cos = sin.to(q.dtype), cos.to(q.dtype)
            if q.is_cuda and q.dtype == torch.bfloat16 and hd % 16 == 0:
                # one pass per tensor, fp32 arithmetic on fp32 (full precision) or bf16 tables, one rounding
                q = _FusedRotary.apply(q, cos, sin).transpose(1, 2)
                k = _FusedRotary.apply(k, cos, sin).transpose(1, 2)
            else:
                q, k = q.transpose(1, 2), k.transpose(1, 2)
                c, s = cos.unsqueeze(1), sin.unsqueeze(1)
                qf, kf = (q.float(), k.float()) if full else (q, k)
                q = (qf * c + _rotate_half(qf) * s).to(q.dtype)
                k = (kf * c + _rotate_half(kf) * s).to(k.dtype)
        else:
            q, k = q.transpose(1, 2), k.transpose(1, 2)
        if n_kv != cfg.n_heads:
            k = k.repeat_interleave(cfg.n_heads // n_kv, dim=1)
            v = v.repeat_interleave(cfg.n_heads // n_kv, dim=1)
        if attention_bias is not None:
            attention_bias = attention_bias[:, :, :T, :T].to(q.dtype)
        att = F.scaled_dot_product_attention(q, k, v, attn_mask=attention_bias,
                                             dropout_p=cfg.attention_dropout if self.training else 0.0,
                                             is_causal=attention_bias is None)
        return att.transpose(1, 2).contiguous().view(B, T, C), None

    @classmethod
    def build(cls, layer_id: int, config, qargs: QuantizationConfig, cache=None):
        if str(getattr(config.block_type, "value", config.block_type)).lower() == "sequential":
            return CoatOLMoSequentialBlock(layer_id, config, qargs, cache)
        raise NotImplementedError(f"Unknown block type: '{config.block_type}'")


class CoatOLMoSequentialBlock(CoatOLMoBlock):
    """``x + MLP(LN(x + Attention(LN(x))))`` on the FP8 stream (coat_olmo.py:910-1076).
    forward(x, qx, sx, ...) -> (x, qx, sx, cache)"""

    def __init__(self, layer_id: int, config, qargs: QuantizationConfig, cache=None):
        super().__init__(layer_id, config, qargs, cache)
        assert not getattr(config, "norm_after", False), "COAT currently does not support PostNorm"
        _check_supported(config)
        head_dim = config.d_model // config.n_heads
        self.fused_dims = (config.d_model, config.effective_n_kv_heads * head_dim,
                           config.effective_n_kv_heads * head_dim)
        self.BeforeAttention = CoatOLMoBeforeAttentionResidual(config, qargs, self.layer_id, self.fused_dims)
        self.AfterAttention = CoatOLMoAfterAttentionResidual(config, qargs, self.layer_id)
        self.MLPResidual = CoatOLMoMLPResidual(config, qargs, self.layer_id, self.hidden_size)

    def reset_parameters(self):
        """The 'mitchell' initialisation of the OLMo-7B configuration (coat_olmo.py:947-990): truncated normals with
        std 1/sqrt(d_model) for the input projections and 1/sqrt(2 * fan_in * (layer + 1)) for the output ones."""
        d = self.config.d_model

        def init(linear, std, cutoff=3.0):
            nn.init.trunc_normal_(linear.weight, mean=0.0, std=std, a=-cutoff * std, b=cutoff * std)
            if linear.bias is not None:
                nn.init.zeros_(linear.bias)

        init(self.AfterAttention.attn_out, 1 / math.sqrt(2 * d * (self.layer_id + 1)))
        init(self.MLPResidual.ff_out, 1 / math.sqrt(2 * self.MLPResidual.ff_out.in_features * (self.layer_id + 1)))
        init(self.BeforeAttention.att_proj, 1 / math.sqrt(d))
        init(self.MLPResidual.ff_proj, 1 / math.sqrt(d))

    def forward(self, x: torch.Tensor, qx: torch.Tensor, sx: torch.Tensor,
                attention_bias: Optional[torch.Tensor] = None, layer_past=None, use_cache: bool = False,
                max_doc_len: Optional[int] = None, cu_doc_lens: Optional[torch.Tensor] = None):
        x, qkv = self.BeforeAttention(x, qx, sx)
        if self.config.clip_qkv is not None:
            qkv = qkv.clamp(min=-self.config.clip_qkv, max=self.config.clip_qkv)
        q, k, v = qkv.split(self.fused_dims, dim=-1)
        att, cache = self.attention(q, k, v, attention_bias, layer_past=layer_past, use_cache=use_cache,
                                    max_doc_len=max_doc_len, cu_doc_lens=cu_doc_lens)
        x, qx, sx = self.AfterAttention(x, att)
        x, qx, sx = self.MLPResidual(x, qx, sx)
        return x, qx, sx, cache


# =====================================================================================================
# The model around the blocks
# =====================================================================================================
class OLMoOutput(NamedTuple):
    logits: torch.Tensor
    attn_key_values: Optional[list]
    hidden_states: Optional[tuple]


class _PlainLayerNorm(nn.Module):
    """LayerNorm without parameters (the OLMo-7B configuration's `layer_norm_type: default`, no affine part)."""

    def __init__(self, eps=1e-5):
        super().__init__()
        self.eps = eps

    def forward(self, x):
        return _plain_layernorm(x, self.eps)


class CoatOLMo(nn.Module):
    """The model around the blocks (coat_olmo.py:1138-1450): `transformer.wte` -> `Coat_quantize_bgn` -> the blocks
    passing the (bf16, FP8 codes, scales) triple -> `Coat_quantize_end` -> `transformer.ln_f` -> `transformer.ff_out`
    (or the tied embedding), with the reference's module names, hence its state-dict keys.  The training model: no KV
    cache, no ALiBi, no document masking, no activation checkpointing (the host trainer's options around the model);
    `attention_mask` (1 = attend) and `attention_bias` are turned into one additive bias as in the reference."""

    def __init__(self, config, qargs: QuantizationConfig, init_params: bool = True):
        super().__init__()
        self.config = config
        self.qargs = qargs
        self._cache = {}
        if getattr(config, "alibi", False):
            raise NotImplementedError("ALiBi is not part of the quantised model")
        if not getattr(config, "rope", True):
            raise NotImplementedError("learned position embeddings are not part of the quantised model")
        vocab = getattr(config, "embedding_size", None) or config.vocab_size
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(vocab, config.d_model, device=_device(config)),
            emb_drop=nn.Dropout(getattr(config, "embedding_dropout", 0.0)),
            ln_f=_PlainLayerNorm(getattr(config, "layer_norm_eps", 1e-5)),
            blocks=nn.ModuleList(CoatOLMoBlock.build(i, config, qargs, self._cache) for i in range(config.n_layers)),
        ))
        if not getattr(config, "weight_tying", False):
            self.transformer.update({"ff_out": nn.Linear(config.d_model, vocab, bias=config.include_bias,
                                                         device=_device(config))})
        self.quantize_input_before_block = Coat_quantize_bgn(qargs)
        self.quantize_output_after_block = Coat_quantize_end(qargs)
        if init_params:
            self.reset_parameters()

    def reset_parameters(self):
        """'mitchell' initialisation (the OLMo-7B configuration): embedding and output std 1/sqrt(d_model), cut at 3 std;
        the blocks as CoatOLMoSequentialBlock.reset_parameters."""
        std = 1 / math.sqrt(self.config.d_model)
        nn.init.trunc_normal_(self.transformer.wte.weight, mean=0.0, std=std, a=-3 * std, b=3 * std)
        if "ff_out" in self.transformer:
            nn.init.trunc_normal_(self.transformer.ff_out.weight, mean=0.0, std=std, a=-3 * std, b=3 * std)
        for block in self.transformer.blocks:
            block.reset_parameters()

    def forward(self, input_ids, input_embeddings=None, attention_mask=None, attention_bias=None,
                past_key_values=None, use_cache: bool = False, last_logits_only: bool = False,
                output_hidden_states: Optional[bool] = None, doc_lens=None, max_doc_lens=None):
        if past_key_values is not None or use_cache:
            raise NotImplementedError("the training model keeps no KV cache")
        if doc_lens is not None or max_doc_lens is not None:
            raise NotImplementedError("document masking needs the host trainer's variable-length attention")
        x = self.transformer.wte(input_ids) if input_embeddings is None else input_embeddings
        batch_size, seq_len = x.shape[:2]
        x = self.transformer.emb_drop(x)
        if attention_mask is not None or attention_bias is not None:
            if attention_bias is None:   # causal
                attention_bias = torch.zeros(1, 1, seq_len, seq_len, dtype=torch.float, device=x.device).masked_fill(
                    torch.ones(seq_len, seq_len, dtype=torch.bool, device=x.device).triu(1), torch.finfo(torch.float).min)
            elif attention_bias.dtype in (torch.int8, torch.bool):
                attention_bias = attention_bias.to(dtype=torch.float)
                attention_bias = attention_bias.masked_fill(attention_bias == 0.0, torch.finfo(torch.float).min)
            attention_bias = attention_bias.reshape((-1, 1) + attention_bias.shape[-2:])[:, :, :seq_len, :seq_len].float()
            if attention_mask is not None:
                pad = (1.0 - attention_mask.to(torch.float).view(batch_size, -1)[:, None, None, :]) * torch.finfo(torch.float).min
                attention_bias = (attention_bias + pad).clamp_min(torch.finfo(torch.float).min)
        hidden = []
        x, qx, sx = self.quantize_input_before_block(x)
        for block in self.transformer.blocks:
            if output_hidden_states:
                hidden.append(x)
            x, qx, sx, _ = block(x, qx, sx, attention_bias=attention_bias)
        x = self.quantize_output_after_block(x, qx, sx)
        if last_logits_only:
            x = x[:, -1, :].unsqueeze(1)
        x = self.transformer.ln_f(x)
        if output_hidden_states:
            hidden.append(x)
        if getattr(self.config, "weight_tying", False):
            logits = F.linear(x, self.transformer.wte.weight, None)
        else:
            logits = self.transformer.ff_out(x)
        if getattr(self.config, "scale_logits", False):
            logits = logits * (1 / math.sqrt(self.config.d_model))
        return OLMoOutput(logits=logits, attn_key_values=None, hidden_states=tuple(hidden) if output_hidden_states else None)

