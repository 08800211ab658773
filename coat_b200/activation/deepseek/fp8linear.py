"""`FP8DeepSeekLinear`: nn.Linear whose training forward / backward run block-scaled FP8 GEMMs, as
coat/activation/deepseek/fp8linear.py:45-126: activations and output gradients in 1 x 128 groups, weights in
128 x 128 blocks, fp32 scales.  Like the reference, the training forward does not add the bias (it is handed
to fp8_deepseek_linear_forward, which ignores it); its gradient is still returned."""
from copy import deepcopy
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd.function import Function

from ..real_quantization._quantize_perblock import fp8_quantize_perblock
from ..real_quantization._quantize_perblock_transpose import fp8_quantize_perblock_transpose
from ..real_quantization._quantize_perblock_transpose_pergroup import fp8_quantize_perblock_transpose_pergroup
from ..real_quantization._quantize_transpose import fp8_quantize_transpose
from .linear import fp8_deepseek_linear_backward, fp8_deepseek_linear_forward


@dataclass
class DefaultArgs:
    fabit: str = "E4M3"
    fwbit: str = "E4M3"
    bobit: str = "E4M3"


def _rows_contiguous(s):
    """[M, G] scales stored with the M index contiguous (stride(0) == 1), the layout the GEMM reads."""
    return s.t().contiguous().t()


class _FP8DeepSeekLinear(Function):
    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, input, weight, bias, args, layer_name):
        x2d = input.reshape(-1, input.shape[-1])
        (q_x, s_x), (q_x_t, s_x_t) = fp8_quantize_transpose(x2d, 128, args.fabit, scale_dtype=torch.float32)
        q_w, s_w = fp8_quantize_perblock(weight, 128, args.fwbit, scale_dtype=torch.float32)
        ctx.save_for_backward(q_x_t, _rows_contiguous(s_x_t), weight, bias)
        ctx.utils = args, layer_name, input.shape, weight.shape
        out = fp8_deepseek_linear_forward(q_x, _rows_contiguous(s_x), q_w, s_w, 0, bias)
        return out.view(*input.shape[:-1], weight.shape[0])

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        q_x_t, s_x_t, weight, bias = ctx.saved_tensors
        args, layer_name, input_shape, weight_shape = ctx.utils
        g2d = grad_output.reshape(-1, grad_output.shape[-1])
        _, (q_g_t, s_g_t), (q_g_pg, s_g_pg) = fp8_quantize_perblock_transpose_pergroup(
            g2d, 128, args.bobit, scale_dtype=torch.float32, only_transposed=True)
        q_w_t, s_w_t = fp8_quantize_perblock_transpose(weight, 128, args.fwbit, scale_dtype=torch.float32,
                                                       only_transposed=True)
        grad_input, grad_weight = fp8_deepseek_linear_backward(q_x_t, s_x_t, q_g_pg, _rows_contiguous(s_g_pg), q_g_t,
                                                               s_g_t, q_w_t, s_w_t)
        grad_bias = g2d.sum(0) if bias is not None else None
        return grad_input.view(input_shape), grad_weight, grad_bias, None, None


class FP8DeepSeekLinear(nn.Linear):
    def __init__(self, in_features, out_features, bias=True, device=None, args=None, layer_idx=0):
        super().__init__(in_features, out_features, bias, device)
        self.args = deepcopy(args if args is not None else DefaultArgs())
        self.layer_idx = layer_idx
        self.layer_name = None

    def forward(self, Input):
        if self.training:
            return _FP8DeepSeekLinear.apply(Input, self.weight, self.bias, self.args, self.layer_name)
        return F.linear(Input, self.weight, self.bias)
