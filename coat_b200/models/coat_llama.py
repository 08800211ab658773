"""The COAT Llama decoder layer on the B200 operators.

Same class names, constructor arguments, forward signatures and data flow as
coat/models/coat_llama.py of the reference: a decoder layer is three autograd blocks that pass a triple
(bf16 hidden states, their 1x16 FP8 codes, the group scales) from one to the next,

    BeforeAttention  (:110-347)  RMSNorm on the FP8 input -> per-tensor FP8 -> q/k/v projections
    attention without linears (:770-1081)  RoPE + causal attention on bf16 q/k/v (torch SDPA here)
    AfterAttention   (:350-488)  per-tensor FP8 of the attention output -> o projection -> residual add
                                 fused with the 1x16 quantisation of the sum
    MLPResidual      (:491-766)  RMSNorm -> gate/up projections with 1x16-quantising epilogue -> SiLU ->
                                 Mul -> down projection -> residual add + 1x16 quantisation

and whose backward passes run the mirrored chain on E5M2 gradients.  What is saved for backward is what
the reference saves (FP8 activations and transposed FP8 copies, never a bf16 activation except the
attention output).  The model around the layers is in coat_llama_model.py; tokenizer and generation
plumbing are not part of this package, and `CoatLlamaConfig` is a plain attribute bag (any object with the same
attributes, e.g. a transformers LlamaConfig carrying `coat_fp8_args`, works).

FP8 tensors cross autograd boundaries viewed as float8_e4m3fn whatever their real format (autograd
insists on matching dtypes; the bytes are untouched), as in the reference.
"""
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..activation.real_quantization import (
    fp8_add_Ifp_Ifp_Ofp_Og16,
    fp8_add_Ifp_Ifp_Ofp_Opt,
    fp8_division,
    fp8_division_transpose,
    fp8_linear_backward,
    fp8_linear_forward,
    fp8_mul_silu_backward,
    fp8_quantize_pertensor,
    fp8_quantize_pertensor_transpose,
    fp8_rmsnorm_backward,
    fp8_rmsnorm_forward,
    fp8_silu_mul_forward,
    fp8_transpose,
)
from ..utils._fp8_quantization_config import QuantizationConfig
from ..utils._fp8_weightcache import FP8CacheWeightModule
from ..utils._fp8manager import FP8Manager


class CoatLlamaConfig:
    """The attributes of the reference's CoatLlamaConfig (a transformers LlamaConfig plus `coat_fp8_args`,
    coat_llama.py:106-107) that the decoder layer and the model read."""
    model_type = "fp8_llama"

    def __init__(self, hidden_size=4096, intermediate_size=11008, num_attention_heads=32, num_key_value_heads=None,
                 head_dim=None, rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=4096,
                 attention_bias=False, attention_dropout=0.0, mlp_bias=False, hidden_act="silu",
                 coat_fp8_args=None, _attn_implementation="sdpa", vocab_size=32000, num_hidden_layers=32,
                 pad_token_id=None, initializer_range=0.02, tie_word_embeddings=False, **kwargs):
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_attention_heads = num_attention_heads
        self.num_key_value_heads = num_key_value_heads or num_attention_heads
        self.head_dim = head_dim or hidden_size // num_attention_heads
        self.rms_norm_eps = rms_norm_eps
        self.rope_theta = rope_theta
        self.max_position_embeddings = max_position_embeddings
        self.attention_bias = attention_bias
        self.attention_dropout = attention_dropout
        self.mlp_bias = mlp_bias
        self.hidden_act = hidden_act
        self.coat_fp8_args = dict(coat_fp8_args or {})
        self._attn_implementation = _attn_implementation
        self.vocab_size = vocab_size
        self.num_hidden_layers = num_hidden_layers
        self.pad_token_id = pad_token_id
        self.initializer_range = initializer_range
        self.tie_word_embeddings = tie_word_embeddings
        for k, v in kwargs.items():
            setattr(self, k, v)


def _fwobits(qargs):
    return {k: getattr(qargs, k) for k in ("fabit", "fwbit", "fobit", "babit", "bwbit", "bobit")}


def _as_e4m3(t):
    return t.view(torch.float8_e4m3fn)


def _forward_weights(origins, codes, scales, qargs, fwbit):
    """Codes of the weights for the forward GEMMs: the cached ones, or (memory-efficient mode) derived from
    the bf16 weights and the cached per-tensor scales."""
    if not qargs.weight_memory_efficient:
        return list(codes)
    assert all(c is None for c in codes), "memory-efficient mode keeps no FP8 weight copies"
    return [fp8_division(w, qargs.group_size, fwbit, s)[0] for w, s in zip(origins, scales)]


def _backward_weight_t(saved, scale, qargs, fwbit):
    """Transposed codes of one weight for dgrad: cached, or derived from the saved bf16 weight."""
    if not qargs.weight_memory_efficient:
        return saved
    return fp8_division_transpose(saved, qargs.group_size, fwbit, scale, only_transposed=True)[0]


# =====================================================================================================
# Before attention: RMSNorm + q/k/v projections
# =====================================================================================================
class _CoatLlamaBeforeAttentionResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, re_x, in_x, in_s, weight1_origin, weight1, weight1_t, weight1_s, weight2_origin, weight2,
                weight2_t, weight2_s, weight3_origin, weight3, weight3_t, weight3_s, rmsnorm_weight, group_size,
                fwobits, layer_id, config, qargs, eps=1e-5):
        if fwobits["fabit"] != "E4M3":
            raise ValueError("fabit should be E4M3")
        in_x = _as_e4m3(in_x)
        ln_x, ln_s, ln_x_t, ln_utils = fp8_rmsnorm_forward(in_x, in_s, rmsnorm_weight, group_size, eps,
                                                           transpose_output_2d=True)
        origins = (weight1_origin, weight2_origin, weight3_origin)
        scales = (weight1_s, weight2_s, weight3_s)
        w = _forward_weights(origins, (weight1, weight2, weight3), scales, qargs, fwobits["fwbit"])
        q, k, v = (fp8_linear_forward(ln_x, ln_s, wi, si, False, group_size) for wi, si in zip(w, scales))

        ctx.save_for_backward(in_x, in_s, ln_x_t, ln_s)
        if qargs.weight_memory_efficient:
            assert weight1_t is None and weight2_t is None and weight3_t is None
            ctx.weight = origins, scales
        else:
            ctx.weight = (weight1_t, weight2_t, weight3_t), scales
        ctx.group_size = group_size
        ctx.ln_utils = ln_utils
        ctx.utils = fwobits, layer_id, config, qargs
        return re_x, q, k, v

    @staticmethod
    def backward(ctx, fp_grad, query_g, key_g, value_g):
        in_x, in_s, ln_x_t, ln_s = ctx.saved_tensors
        saved_w, scales = ctx.weight
        group_size = ctx.group_size
        rms_weight, rstd, num_warps = ctx.ln_utils
        fwobits, layer_id, config, qargs = ctx.utils

        dgrads, wgrads = [], []
        for g, saved, s_w in zip((query_g, key_g, value_g), saved_w, scales):
            # dgrad wants the gradient as it is, wgrad its transposed copy: one quantisation writes both
            qg, qg_s, qg_t = fp8_quantize_pertensor_transpose(g, group_size, fwobits["babit"],
                                                              transpose_output_2d=True, stochastic=False)
            w_t = _backward_weight_t(saved, s_w, qargs, fwobits["fwbit"])
            dx, dw = fp8_linear_backward(ln_x_t, ln_s, qg, qg_s, qg_t, w_t, s_w, group_size)
            dgrads.append(dx)
            wgrads.append(dw)
        # the three input gradients are summed (in bf16, left to right, as `a + b + c` would) inside the norm's
        # backward kernel
        in_g, rms_weight_grad = fp8_rmsnorm_backward(in_x, in_s, dgrads[0], rms_weight, rstd, group_size, num_warps,
                                                     more_g=(dgrads[1], dgrads[2]))
        # residual gradient + norm gradient, and the per-tensor FP8 copy for the block below
        re_g, (in_g, in_sg, in_sg_g16) = fp8_add_Ifp_Ifp_Ofp_Opt(fp_grad, in_g, group_size, fwobits["babit"],
                                                                 stochastic=False)
        # in_sg_g16 (one scale per group) rather than the tensor scale goes back: its shape must match the
        # forward's scale input; the receiver takes its maximum
        return (re_g, _as_e4m3(in_g), in_sg_g16,
                wgrads[0], None, None, None, wgrads[1], None, None, None, wgrads[2], None, None, None,
                rms_weight_grad, None, None, None, None, None, None)


class CoatLlamaBeforeAttentionResidual(FP8CacheWeightModule):
    """Residual pass-through, RMSNorm and the q/k/v projections."""

    def __init__(self, config, qargs: QuantizationConfig, layer_idx: Optional[int] = None):
        super().__init__(config, qargs, layer_idx)
        self.qargs = qargs
        self.fwobits = _fwobits(qargs)
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = getattr(config, "head_dim", None) or self.hidden_size // self.num_heads
        self.num_key_value_heads = config.num_key_value_heads
        bias = getattr(config, "attention_bias", False)
        self.q_proj = nn.Linear(self.hidden_size, self.num_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)

    def forward(self, re_x, x, s, rmsnorm_weight):
        if not self.training:
            x = F.rms_norm(re_x, rmsnorm_weight.shape, rmsnorm_weight)
            return re_x, self.q_proj(x), self.k_proj(x), self.v_proj(x)
        args = []
        with torch.no_grad():
            for name in ("q_proj", "k_proj", "v_proj"):
                weight = getattr(self, name).weight
                prepared = self.prepare_weight(weight, name, FP8Manager.is_first_microbatch)
                if self.qargs.weight_memory_efficient:
                    args += [weight, None, None, prepared]
                else:
                    args += [weight, prepared[0], prepared[1], prepared[2]]
        return _CoatLlamaBeforeAttentionResidual.apply(re_x, x, s, *args, rmsnorm_weight, self.qargs.group_size,
                                                       self.fwobits, self.layer_id, self.config, self.qargs)


# =====================================================================================================
# After attention: o projection + residual
# =====================================================================================================
class _CoatLlamaAfterAttentionResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, re_x, flash_x, weight4_origin, weight4, weight4_t, weight4_s, group_size, fwobits, layer_id,
                config, qargs):
        flash_qx, flash_s, _ = fp8_quantize_pertensor(flash_x, group_size, fwobits["fabit"])
        (weight4,) = _forward_weights((weight4_origin,), (weight4,), (weight4_s,), qargs, fwobits["fwbit"])
        fc4_x = fp8_linear_forward(flash_qx, flash_s, weight4, weight4_s, False, group_size)
        fp_x, (out_x, out_s) = fp8_add_Ifp_Ifp_Ofp_Og16(re_x, fc4_x, flash_qx.dtype, group_size)

        # the bf16 attention output is kept (not its FP8 copy): backward re-derives the transposed codes
        ctx.save_for_backward(flash_x, flash_s)
        if qargs.weight_memory_efficient:
            assert weight4_t is None
            ctx.weight = weight4_origin, weight4_s
        else:
            ctx.weight = weight4_t, weight4_s
        ctx.group_size = group_size
        ctx.utils = fwobits, layer_id, config, qargs
        return fp_x, _as_e4m3(out_x), out_s

    @staticmethod
    def backward(ctx, fp_grad, out_g, out_gs):
        flash_x, flash_s = ctx.saved_tensors
        saved_w, weight4_s = ctx.weight
        group_size = ctx.group_size
        fwobits, layer_id, config, qargs = ctx.utils
        if fwobits["babit"] != "E5M2":
            raise ValueError("babit should be E5M2")
        out_g = out_g.view(torch.float8_e5m2)
        out_gs_max = out_gs.max()

        out_g_t = fp8_transpose(out_g, transpose_output_2d=True)
        flash_x_t, flash_s = fp8_division_transpose(flash_x, group_size, fwobits["fabit"], flash_s, stochastic=False,
                                                    only_transposed=True)
        weight4_t = _backward_weight_t(saved_w, weight4_s, qargs, fwobits["fwbit"])
        fc4_g, attn_out_wg = fp8_linear_backward(flash_x_t, flash_s, out_g, out_gs_max, out_g_t, weight4_t, weight4_s,
                                                 group_size)
        return fp_grad, fc4_g, attn_out_wg, None, None, None, None, None, None, None, None


class CoatLlamaAfterAttentionResidual(FP8CacheWeightModule):
    """The attention output projection and the residual add."""

    def __init__(self, config, qargs: QuantizationConfig, layer_id):
        super().__init__(config, qargs, layer_id)
        self.qargs = qargs
        self.fwobits = _fwobits(qargs)
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = getattr(config, "head_dim", None) or self.hidden_size // self.num_heads
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, self.hidden_size,
                                bias=getattr(config, "attention_bias", False))

    def forward(self, re_x, in_x):
        if not self.training:
            return re_x + self.o_proj(in_x), None, None
        with torch.no_grad():
            prepared = self.prepare_weight(self.o_proj.weight, "o_proj", FP8Manager.is_first_microbatch)
        if self.qargs.weight_memory_efficient:
            w, w_t, w_s = None, None, prepared
        else:
            w, w_t, w_s = prepared
        return _CoatLlamaAfterAttentionResidual.apply(re_x, in_x, self.o_proj.weight, w, w_t, w_s,
                                                      self.qargs.group_size, self.fwobits, self.layer_id, self.config,
                                                      self.qargs)


# =====================================================================================================
# MLP: RMSNorm + gate/up + SiLU * up + down + residual
# =====================================================================================================
class _CoatLlamaMLPResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, re_x, in_x, in_s, weight1_origin, weight1, weight1_t, weight1_s, weight2_origin, weight2,
                weight2_t, weight2_s, weight3_origin, weight3, weight3_t, weight3_s, rmsnorm_weight, group_size,
                fwobits, layer_id, config, qargs, eps=1e-5):
        if fwobits["fabit"] != "E4M3":
            raise ValueError("fabit should be E4M3")
        in_x = _as_e4m3(in_x)
        ln_x, ln_s, ln_x_t, ln_utils = fp8_rmsnorm_forward(in_x, in_s, rmsnorm_weight, group_size, eps,
                                                           transpose_output_2d=True)
        origins = (weight1_origin, weight2_origin, weight3_origin)
        scales = (weight1_s, weight2_s, weight3_s)
        w_gate, w_up, w_down = _forward_weights(origins, (weight1, weight2, weight3), scales, qargs, fwobits["fwbit"])

        # gate / up projections leave the GEMM already quantised in 1x16 groups
        gate_x, gate_s = fp8_linear_forward(ln_x, ln_s, w_gate, weight1_s, True, group_size)
        up_x, up_s = fp8_linear_forward(ln_x, ln_s, w_up, weight2_s, True, group_size)
        # (one kernel for fp8_silu_forward followed by fp8_mul_forward: same bits)
        (silu_x, silu_s), (mul_x, mul_s, mul_x_t) = fp8_silu_mul_forward(gate_x, gate_s, up_x, up_s, group_size,
                                                                         transpose_output_2d=True)
        fc3_x = fp8_linear_forward(mul_x, mul_s, w_down, weight3_s, False, group_size)
        fp_x, (out_x, out_s) = fp8_add_Ifp_Ifp_Ofp_Og16(re_x, fc3_x, mul_x.dtype, group_size)

        ctx.save_for_backward(in_x, in_s, ln_x_t, ln_s, gate_x, gate_s, up_x, up_s, silu_x, silu_s, mul_x_t, mul_s)
        if qargs.weight_memory_efficient:
            assert weight1_t is None and weight2_t is None and weight3_t is None
            ctx.weight = origins, scales
        else:
            ctx.weight = (weight1_t, weight2_t, weight3_t), scales
        ctx.group_size = group_size
        ctx.ln_utils = ln_utils
        ctx.utils = fwobits, layer_id, config, qargs
        return fp_x, _as_e4m3(out_x), out_s

    @staticmethod
    def backward(ctx, fp_grad, out_g, out_gs):
        in_x, in_s, ln_x_t, ln_s, gate_x, gate_s, up_x, up_s, silu_x, silu_s, mul_x_t, mul_s = ctx.saved_tensors
        (saved_gate, saved_up, saved_down), (weight1_s, weight2_s, weight3_s) = ctx.weight
        group_size = ctx.group_size
        rms_weight, rstd, num_warps = ctx.ln_utils
        fwobits, layer_id, config, qargs = ctx.utils
        if fwobits["babit"] != "E5M2":
            raise ValueError("babit should be E5M2")
        out_g = out_g.view(torch.float8_e5m2)
        out_gs_max = out_gs.max()

        # down projection
        out_g_t = fp8_transpose(out_g, transpose_output_2d=True)
        w_down_t = _backward_weight_t(saved_down, weight3_s, qargs, fwobits["fwbit"])
        fc3_g, weight3_grad = fp8_linear_backward(mul_x_t, mul_s, out_g, out_gs_max, out_g_t, w_down_t, weight3_s,
                                                  group_size)
        del out_g, out_g_t, w_down_t

        # Mul (1: towards the gate branch, bf16; 2: towards up, per-tensor FP8 + transposed copy), then SiLU
        # (one kernel for fp8_mul_backward followed by fp8_silu_backward: same bits, no bf16 round trip between them)
        (mul_g2, mul_gs2, mul_g2_t), (silu_g, silu_gs, silu_g_t) = fp8_mul_silu_backward(
            silu_x, silu_s, up_x, up_s, gate_x, gate_s, fc3_g, group_size, fwobits["babit"])

        # gate / up projections
        w_gate_t = _backward_weight_t(saved_gate, weight1_s, qargs, fwobits["fwbit"])
        w_up_t = _backward_weight_t(saved_up, weight2_s, qargs, fwobits["fwbit"])
        fc1_g, weight1_grad = fp8_linear_backward(ln_x_t, ln_s, silu_g, silu_gs, silu_g_t, w_gate_t, weight1_s,
                                                  group_size)
        fc2_g, weight2_grad = fp8_linear_backward(ln_x_t, ln_s, mul_g2, mul_gs2, mul_g2_t, w_up_t, weight2_s,
                                                  group_size)
        in_g, rms_weight_grad = fp8_rmsnorm_backward(in_x, in_s, fc1_g, rms_weight, rstd, group_size, num_warps,
                                                     more_g=(fc2_g,))   # fc1_g + fc2_g, summed in the kernel
        re_g, (in_g, in_sg, in_sg_g16) = fp8_add_Ifp_Ifp_Ofp_Opt(fp_grad, in_g, group_size, fwobits["babit"],
                                                                 stochastic=False)
        return (re_g, _as_e4m3(in_g), in_sg_g16,
                weight1_grad, None, None, None, weight2_grad, None, None, None, weight3_grad, None, None, None,
                rms_weight_grad, None, None, None, None, None, None)


class CoatLlamaMLPResidual(FP8CacheWeightModule):
    """Residual, RMSNorm and the gated MLP."""

    def __init__(self, config, qargs: QuantizationConfig, layer_id, hidden_size: int):
        super().__init__(config, qargs, layer_id)
        self.qargs = qargs
        self.fwobits = _fwobits(qargs)
        self.config = config
        self.hidden_size = config.hidden_size
        self.intermediate_size = config.intermediate_size
        bias = getattr(config, "mlp_bias", False)
        self.gate_proj = nn.Linear(self.hidden_size, self.intermediate_size, bias=bias)
        self.up_proj = nn.Linear(self.hidden_size, self.intermediate_size, bias=bias)
        self.down_proj = nn.Linear(self.intermediate_size, self.hidden_size, bias=bias)
        assert getattr(config, "hidden_act", "silu") == "silu", "We only support silu activation currently"

    def forward(self, re_x, x, s, rmsnorm_weight):
        if not self.training:
            h = F.rms_norm(re_x, rmsnorm_weight.shape, rmsnorm_weight)
            return re_x + self.down_proj(F.silu(self.gate_proj(h)) * self.up_proj(h)), None, None
        args = []
        with torch.no_grad():
            for name in ("gate_proj", "up_proj", "down_proj"):
                weight = getattr(self, name).weight
                prepared = self.prepare_weight(weight, name, FP8Manager.is_first_microbatch)
                if self.qargs.weight_memory_efficient:
                    args += [weight, None, None, prepared]
                else:
                    args += [weight, prepared[0], prepared[1], prepared[2]]
        return _CoatLlamaMLPResidual.apply(re_x, x, s, *args, rmsnorm_weight, self.qargs.group_size, self.fwobits,
                                           self.layer_id, self.config, self.qargs)


# =====================================================================================================
# Attention without the linear layers
# =====================================================================================================
def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


class _FusedRotary(torch.autograd.Function):
    """y = x * cos + rotate_half(x) * sin on bf16 [B, S, H, D] in one kernel (coat_rope_bf16, or its variant for fp32
    cos / sin tables); the backward pass is the same kernel with the transposed rotation."""

    @staticmethod
    def _run(x4, cos, sin, backward):
        from .. import _lib
        B, S, H, D = x4.shape
        y = torch.empty((B, S, H, D), dtype=x4.dtype, device=x4.device)
        with torch.cuda.device(x4.device):
            fn = _lib.lib().coat_rope_bf16 if cos.dtype == torch.bfloat16 else _lib.lib().coat_rope_bf16_f32tables
            rc = fn(x4.data_ptr(), x4.stride(0), x4.stride(1), x4.stride(2), cos.data_ptr(), sin.data_ptr(),
                    y.data_ptr(), B, S, H, D, 0 if cos.shape[0] == 1 else cos.stride(0), int(backward),
                    _lib.stream_ptr(x4.device))
        _lib.check(rc, "rope_bf16")
        return y

    @staticmethod
    def forward(ctx, x4, cos, sin):
        ctx.save_for_backward(cos, sin)
        return _FusedRotary._run(x4, cos, sin, False)

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        if dy.stride(3) != 1 or any(st % 8 for st in dy.stride()[:3]):
            dy = dy.contiguous()
        return _FusedRotary._run(dy, cos, sin, True), None, None


def _fused_rotary_ok(x, cos, sin):
    return (x.is_cuda and x.dtype == torch.bfloat16 and cos.dtype == torch.bfloat16 and sin.dtype == torch.bfloat16
            and cos.dim() == 3 and cos.is_contiguous() and sin.is_contiguous() and cos.shape == sin.shape
            and cos.shape[0] in (1, x.shape[0]) and x.shape[-1] % 16 == 0)


def llama_rotary_embeddings(position_ids, head_dim, rope_theta, dtype):
    """cos / sin of shape [batch, seq, head_dim] for integer positions [batch, seq] (default Llama RoPE)."""
    inv_freq = 1.0 / (rope_theta ** (torch.arange(0, head_dim, 2, device=position_ids.device, dtype=torch.float32)
                                    / head_dim))
    freqs = position_ids.to(torch.float32)[..., None] * inv_freq
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


class LlamaSdpaAttentionWithoutLinear(nn.Module):
    """RoPE + scaled-dot-product attention on already projected q/k/v of shape [batch, seq, heads*head_dim]
    (coat_llama.py:981-1081 with torch's SDPA kernels; no KV cache: this is the training layer)."""

    def __init__(self, config, layer_idx: Optional[int] = None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = getattr(config, "head_dim", None) or self.hidden_size // self.num_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.rope_theta = getattr(config, "rope_theta", 10000.0)
        self.attention_dropout = getattr(config, "attention_dropout", 0.0)
        self.is_causal = True

    def forward(self, query_states, key_states, value_states, attention_mask=None, position_ids=None,
                past_key_value=None, output_attentions=False, use_cache=False, cache_position=None,
                position_embeddings=None, **kwargs):
        if output_attentions or use_cache or past_key_value is not None:
            raise NotImplementedError("the training layer returns no attention weights and keeps no KV cache")
        bsz, q_len, _ = query_states.size()
        q = query_states.view(bsz, q_len, self.num_heads, self.head_dim)
        k = key_states.view(bsz, q_len, self.num_key_value_heads, self.head_dim)
        v = value_states.view(bsz, q_len, self.num_key_value_heads, self.head_dim).transpose(1, 2)
        if position_embeddings is None:
            if position_ids is None:
                position_ids = torch.arange(q_len, device=q.device)[None, :]
            position_embeddings = llama_rotary_embeddings(position_ids, self.head_dim, self.rope_theta, q.dtype)
        cos, sin = position_embeddings
        if _fused_rotary_ok(q, cos, sin):
            q = _FusedRotary.apply(q, cos, sin).transpose(1, 2)
            k = _FusedRotary.apply(k, cos, sin).transpose(1, 2)
        else:   # other dtypes / devices: the eager form
            q, k = q.transpose(1, 2), k.transpose(1, 2)
            cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
            q = q * cos + _rotate_half(q) * sin
            k = k * cos + _rotate_half(k) * sin
        if self.num_key_value_groups > 1:
            k = k.repeat_interleave(self.num_key_value_groups, dim=1)
            v = v.repeat_interleave(self.num_key_value_groups, dim=1)
        causal = attention_mask is None and q_len > 1
        out = F.scaled_dot_product_attention(q, k, v, attn_mask=attention_mask,
                                             dropout_p=self.attention_dropout if self.training else 0.0,
                                             is_causal=causal)
        return out.transpose(1, 2).contiguous().view(bsz, q_len, -1), None, None


COAT_LLAMA_ATTENTION_CLASSES = {
    "eager": LlamaSdpaAttentionWithoutLinear,
    "sdpa": LlamaSdpaAttentionWithoutLinear,
}


class LlamaRMSNorm(nn.Module):
    """Holder of the norm weight (the fused blocks apply the norm themselves); plain RMSNorm when called."""

    def __init__(self, hidden_size, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, hidden_states):
        return F.rms_norm(hidden_states, self.weight.shape, self.weight, self.variance_epsilon)


class CoatLlamaDecoderLayer(nn.Module):
    """coat_llama.py:1084-1181.  forward((hidden, FP8 codes, scales), ...) -> (((hidden, codes, scales),),)"""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        impl = getattr(config, "_attn_implementation", "sdpa")
        self.self_attn = COAT_LLAMA_ATTENTION_CLASSES.get(impl, LlamaSdpaAttentionWithoutLinear)(
            config=config, layer_idx=layer_idx)
        self.qargs = QuantizationConfig(**config.coat_fp8_args)
        self.BeforeAttention = CoatLlamaBeforeAttentionResidual(config, self.qargs, layer_idx)
        self.AfterAttention = CoatLlamaAfterAttentionResidual(config, self.qargs, layer_idx)
        self.MLPResidual = CoatLlamaMLPResidual(config, self.qargs, layer_idx, self.hidden_size)
        self.input_layernorm = LlamaRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = LlamaRMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, hidden_states: torch.Tensor, quant_hidden_states: torch.Tensor,
                scale_hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.LongTensor] = None, past_key_value=None,
                output_attentions: Optional[bool] = False, use_cache: Optional[bool] = False,
                cache_position: Optional[torch.LongTensor] = None,
                position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, **kwargs):
        residual, q, k, v = self.BeforeAttention(hidden_states, quant_hidden_states, scale_hidden_states,
                                                 self.input_layernorm.weight)
        hidden_states, attn_weights, present = self.self_attn(
            query_states=q, key_states=k, value_states=v, attention_mask=attention_mask, position_ids=position_ids,
            past_key_value=past_key_value, output_attentions=output_attentions, use_cache=use_cache,
            cache_position=cache_position, position_embeddings=position_embeddings, **kwargs)
        hidden_states, quant_hidden_states, scale_hidden_states = self.AfterAttention(residual, hidden_states)
        hidden_states, quant_hidden_states, scale_hidden_states = self.MLPResidual(
            hidden_states, quant_hidden_states, scale_hidden_states, self.post_attention_layernorm.weight)
        outputs = ((hidden_states, quant_hidden_states, scale_hidden_states),)
        if output_attentions:
            outputs += (attn_weights,)
        if use_cache:
            outputs += (present,)
        return outputs
