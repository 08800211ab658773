"""FP8Linear: nn.Linear whose training forward / backward run on FP8 tensor cores.

Mirror of coat/activation/real_quantization/fp8linear.py (FP8Linear :41-62, QuantLinearTE :64-110):
per-tensor E4M3 quantisation (with the transposed copy for the backward GEMMs) of input and weight,
forward GEMM in FP8, per-tensor E5M2 quantisation of the output gradient, dgrad and wgrad GEMMs in FP8."""
import os
from copy import deepcopy
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd.function import Function

from ._quantize_pertensor_transpose import fp8_quantize_pertensor_transpose
from .linear import fp8_linear_backward, fp8_linear_forward


@dataclass
class DefaultArgs:
    fabit: str = "E4M3"
    fwbit: str = "E4M3"
    bobit: str = "E5M2"


class FP8Linear(nn.Linear):
    def __init__(self, in_features, out_features, bias=True, device=None, args=None, layer_idx=0):
        super().__init__(in_features, out_features, bias, device)
        if args is None:
            args = DefaultArgs()
        self.args = deepcopy(args)
        if int(os.environ.get("LOCAL_RANK", "0")) == 0 and os.environ.get("COAT_B200_VERBOSE"):
            print(f"[qlinear debug] Apply QLinear, {layer_idx}")
        self.layer_idx = layer_idx
        self.layer_name = None

    def forward(self, Input):
        if self.training:
            return QuantLinearTE.apply(Input, self.weight, self.bias, self.args, self.layer_name)
        return F.linear(Input, self.weight, self.bias)


class QuantLinearTE(Function):
    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.bfloat16)
    def forward(ctx, input, weight, bias, args, layer_name):
        Qinput, Iscale, Qinput_t = fp8_quantize_pertensor_transpose(input, 16, args.fabit, transpose_output_2d=True)
        Qweight, Wscale, Qweight_t = fp8_quantize_pertensor_transpose(weight, 16, args.fwbit, transpose_output_2d=True)
        ctx.saved = Qinput_t, Iscale, Qweight_t, Wscale, bias, args, layer_name
        return fp8_linear_forward(Qinput, Iscale, Qweight, Wscale, False, 0, bias)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        Qinput_t, Iscale, Qweight_t, Wscale, bias, args, layer_name = ctx.saved
        Qgrad_output, Gscale, Qgrad_output_t = fp8_quantize_pertensor_transpose(
            grad_output, 16, args.bobit, stochastic=False, transpose_output_2d=True)
        grad_input, grad_weight = fp8_linear_backward(
            Qinput_t, Iscale, Qgrad_output, Gscale, Qgrad_output_t, Qweight_t, Wscale, 16, bias,
            stochastic=False, dgrad_quantize=False)
        grad_bias = grad_output.reshape(-1, grad_output.shape[-1]).sum(0) if bias is not None else None
        return grad_input, grad_weight, grad_bias, None, None
