"""FP8Linear: nn.Linear whose training forward / backward run on the FP8 tensor cores
(coat/activation/real_quantization/fp8linear.py: FP8Linear :41-62, QuantLinearTE :64-110).

Forward: input and weight are quantised per tensor to `fabit` / `fwbit` together with their transposed
copies (the backward GEMMs need K-major operands), one FP8 GEMM.  Backward: the output gradient is quantised
per tensor to `bobit` (E5M2 by default) with its transpose, then the dgrad and wgrad GEMMs.  Outside
training it is a plain nn.Linear."""
import os
from copy import deepcopy
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd.function import Function

from ._quantize_pertensor_transpose import fp8_quantize_pertensor_transpose as _quantize_both_ways
from .linear import fp8_linear_backward, fp8_linear_forward

_GROUP = 16   # group size handed to the quantizers (their per-tensor scale is the maximum over these groups)


@dataclass
class DefaultArgs:
    fabit: str = "E4M3"
    fwbit: str = "E4M3"
    bobit: str = "E5M2"


class QuantLinearTE(Function):
    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.bfloat16)
    def forward(ctx, input, weight, bias, args, layer_name):
        q_in, s_in, q_in_t = _quantize_both_ways(input, _GROUP, args.fabit, transpose_output_2d=True)
        q_w, s_w, q_w_t = _quantize_both_ways(weight, _GROUP, args.fwbit, transpose_output_2d=True)
        ctx.saved = q_in_t, s_in, q_w_t, s_w, bias, args
        return fp8_linear_forward(q_in, s_in, q_w, s_w, False, 0, bias)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        q_in_t, s_in, q_w_t, s_w, bias, args = ctx.saved
        q_g, s_g, q_g_t = _quantize_both_ways(grad_output, _GROUP, args.bobit, stochastic=False,
                                              transpose_output_2d=True)
        d_input, d_weight = fp8_linear_backward(q_in_t, s_in, q_g, s_g, q_g_t, q_w_t, s_w, _GROUP, bias,
                                                stochastic=False, dgrad_quantize=False)
        d_bias = None if bias is None else grad_output.reshape(-1, grad_output.shape[-1]).sum(0)
        return d_input, d_weight, d_bias, None, None


class FP8Linear(nn.Linear):
    def __init__(self, in_features, out_features, bias=True, device=None, args=None, layer_idx=0):
        super().__init__(in_features, out_features, bias, device)
        self.args = deepcopy(DefaultArgs() if args is None else args)
        self.layer_idx = layer_idx
        self.layer_name = None
        if os.environ.get("COAT_B200_VERBOSE") and int(os.environ.get("LOCAL_RANK", "0")) == 0:
            print(f"[qlinear debug] Apply QLinear, {layer_idx}")

    def forward(self, Input):
        if not self.training:
            return F.linear(Input, self.weight, self.bias)
        return QuantLinearTE.apply(Input, self.weight, self.bias, self.args, self.layer_name)
