"""Entry and exit of the FP8 activation stream of a model, as
coat/activation/real_quantization/func_quantize.py:24-110.

`Coat_quantize_bgn` turns the bf16 hidden states into the triple (bf16, 1xQB FP8 codes, scales) that
the decoder layers pass along; its backward hands the bf16 gradient through.  `Coat_quantize_end`
drops the FP8 copy in forward; its backward produces the (bf16, per-tensor FP8, 1xQB scales) triple of
the gradient stream.  FP8 tensors cross autograd boundaries viewed as float8_e4m3fn whatever their
real format, as in the reference (autograd wants matching dtypes, the bytes are untouched)."""
from copy import deepcopy

import torch
import torch.nn as nn

from ._quantize import fp8_quantize
from ._quantize_pertensor import fp8_quantize_pertensor


class Coat_quantize_bgn_func(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, group_size, fp8type):
        q, s = fp8_quantize(input, group_size, fp8type)
        return input, q.view(torch.float8_e4m3fn), s

    @staticmethod
    def backward(ctx, grad_output, Qgrad_output, Gscale):
        return grad_output, None, None


class Coat_quantize_end_func(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, Qinput, Iscale, group_size, fp8type):
        ctx.saved = group_size, fp8type
        return input

    @staticmethod
    def backward(ctx, grad_output):
        group_size, fp8type = ctx.saved
        q, _, s_g16 = fp8_quantize_pertensor(grad_output, group_size, fp8type, stochastic=False)
        return grad_output, q.view(torch.float8_e4m3fn), s_g16, None, None


class Coat_quantize_bgn(nn.Module):
    def __init__(self, args=None, layer_type=""):
        super().__init__()
        self.args = deepcopy(args)
        self.fp8type = self.args.fabit
        self.layer_type = layer_type

    def forward(self, input):
        if self.training:
            return Coat_quantize_bgn_func.apply(input, self.args.group_size, self.fp8type)
        return input, None, None


class Coat_quantize_end(nn.Module):
    def __init__(self, args=None, layer_type=""):
        super().__init__()
        self.args = deepcopy(args)
        self.fp8type = self.args.babit
        self.layer_type = layer_type

    def forward(self, input, Qinput, Iscale):
        if self.training:
            return Coat_quantize_end_func.apply(input, Qinput, Iscale, self.args.group_size, self.fp8type)
        return input
