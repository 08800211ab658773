"""CPU restatement of the reference's fused quantize-on-save operators in torch fp32 (TEST
INFRASTRUCTURE ONLY).  Each function follows the arithmetic of one wrapper + Triton kernel of
coat/activation/real_quantization/ (silu_fwd.py:100-118, silu_bwd.py:112-137 and :214-224,
gelu_fwd.py:100-118, gelu_bwd.py:112-140, mul_fwd.py:101-127 and :233-238, mul_bwd.py:117-152,
add_fwd.py:92-121, add_bwd.py:92-113 and :185-190, func_rmsnorm.py:77-110 and :152-183), including
that the bf16 intermediate, not the fp32 value, is what the per-tensor division divides, while the
group scales and their maximum come from the fp32 values.

Parity level against the GPU kernels: transcendental functions (exp, erf) come from the host libm here
and libdevice there, and the GPU divides with div.full.f32, so codes agree except at rounding
boundaries and bf16 intermediates to one bf16 ulp; RMSNorm sums in a different order.  The tests state
the resulting tolerances.
"""
import math

import torch

from .quant import FP8_MAX, _dt, cast_fp8, fp8_division, fp8_quantize, group_scales


def dequant(q, s, QB):
    M, N = q.shape
    return (q.float().reshape(M, N // QB, QB) * s.float().unsqueeze(-1)).reshape(M, N)


def _scales_and_max(v, QB, fp8type, scale_dtype=torch.bfloat16):
    s = group_scales(v, QB, fp8type).to(scale_dtype)
    return s, s.max()


def silu_forward(x, s_x, QB):
    v = dequant(x, s_x, QB)
    y = (1.0 / (1.0 + torch.exp(-v))) * v
    return fp8_quantize(y, QB, x.dtype, s_x.dtype)


def silu_backward_value(x, s_x, g, QB):
    v = dequant(x, s_x, QB)
    sg = 1.0 / (1.0 + torch.exp(-v))
    return (sg + v * sg * (1 - sg)) * g.float()


def gelu_forward_value(x, s_x, QB):
    v = dequant(x, s_x, QB)
    return ((1.0 + torch.erf(v / math.sqrt(2.0))) / 2) * v


def gelu_backward_value(x, s_x, g, QB):
    v = dequant(x, s_x, QB)
    cdf = (1.0 + torch.erf(v / math.sqrt(2.0))) / 2
    return (cdf + v * torch.exp(-v * v / 2) / math.sqrt(2 * math.pi)) * g.float()


def per_tensor_from_value(v, QB, fp8type, scale_dtype=torch.bfloat16, transposed=True):
    """bf16 intermediate, group scales from the fp32 value, their max, division of the bf16 by it."""
    y = v.to(torch.bfloat16)
    s_y, s_max = _scales_and_max(v, QB, fp8type, scale_dtype)
    q = fp8_division(y, fp8type, s_max)
    q_t = q.view(torch.uint8).t().contiguous().view(q.dtype) if transposed else None
    return y, s_y, s_max, q, q_t


def mul_forward_value(x1, s1, x2, s2, QB):
    return dequant(x1, s1, QB) * dequant(x2, s2, QB)


def mul_backward_values(x1, s1, x2, s2, g, QB):
    return g.float() * dequant(x2, s2, QB), g.float() * dequant(x1, s1, QB)


def add_forward(x1, x2, fp8type, QB):
    v = x1.float() + x2.float()
    q, s = fp8_quantize(v, QB, fp8type, torch.bfloat16)
    return v.to(torch.bfloat16), (q, s)


def rmsnorm_forward_value(x, s_x, w, QB, eps):
    v = dequant(x, s_x, QB)
    var = (v * v).sum(dim=1, keepdim=True) / v.shape[1]
    rstd = 1 / torch.sqrt(var + eps)
    return (v * rstd) * w.float(), rstd.flatten()


def rmsnorm_row_scales(y_value, fp8type):
    amax = y_value.abs().amax(dim=1)
    return ((amax + torch.tensor(1e-10)) / FP8_MAX[_dt(fp8type)]).to(torch.bfloat16)


def rmsnorm_backward(x, s_x, g, w, rstd, QB):
    v = dequant(x, s_x, QB)
    xhat = v * rstd.unsqueeze(1)
    wdy = w.float() * g.float()
    c1 = (xhat * wdy).sum(dim=1, keepdim=True) / v.shape[1]
    dx = ((wdy - xhat * c1) * rstd.unsqueeze(1)).to(torch.bfloat16)
    dw = (g.float() * xhat).sum(dim=0)
    return dx, dw


# ---- LayerNorm (func_layernorm_noparam.py:54-186, func_layernorm_param.py:54-200) ---------------------
def layernorm_forward_value(x, s_x, w, b, QB, eps):
    """-> (fp32 value before the per-tensor quantisation, mean, rstd).  w = b = None: no affine part."""
    v = dequant(x, s_x, QB)
    n = v.shape[1]
    mean = v.sum(dim=1, keepdim=True) / n
    d = v - mean
    # the reference's kernels pad the row with zeros to the next power of two and do not mask the padding out of the
    # squared deviations (func_layernorm_noparam.py:86-94, func_layernorm_param.py:86-94): each padded element adds
    # mean^2.  Rows whose length is a power of two are unaffected.
    n2 = 1 << max(4, (n - 1).bit_length())
    var = ((d * d).sum(dim=1, keepdim=True) + (n2 - n) * mean * mean) / n
    rstd = 1 / torch.sqrt(var + eps)
    y = d * rstd
    if w is not None:
        y = y * w.float() + b.float()
    return y, mean.flatten(), rstd.flatten()


def layernorm_backward(x, s_x, g, w, mean, rstd, QB):
    """-> (dx bf16, dw, db); dw = db = None without weight."""
    v = dequant(x, s_x, QB)
    n = v.shape[1]
    xhat = (v - mean.unsqueeze(1)) * rstd.unsqueeze(1)
    wdy = g.float() if w is None else w.float() * g.float()
    c1 = (xhat * wdy).sum(dim=1, keepdim=True) / n
    c2 = wdy.sum(dim=1, keepdim=True) / n
    dx = ((wdy - (xhat * c1 + c2)) * rstd.unsqueeze(1)).to(torch.bfloat16)
    if w is None:
        return dx, None, None
    return dx, (g.float() * xhat).sum(dim=0), g.float().sum(dim=0)
