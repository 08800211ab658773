"""FP8 matmul and the linear forward / backward built on it: same names, arguments and return values as
coat/activation/real_quantization/linear.py (fp8matmul :172-250, fp8_linear_forward :253-258,
fp8_linear_backward :272-302).  The work is one tcgen05 GEMM per call behind the C ABI."""
import torch

from ... import _lib
from ._ops import _call, _flags


def fp8matmul(a, b, output_quantize, scale_a, scale_b, QB, bias=None, stochastic=False, *, flags=None):
    """a: [M,K] (or [B,S,K]) FP8, contiguous.  b: [K,N] FP8 view whose K dimension is contiguous, i.e. the
    `.t()` of a contiguous [N,K] matrix, as every call site of the reference passes it."""
    if stochastic:
        raise NotImplementedError("stochastic rounding is not provided")
    batched = a.dim() == 3
    if batched:
        BS = a.shape[0]
        a = a.reshape(-1, a.shape[2])
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.is_contiguous(), "Matrix A must be contiguous"
    if not a.is_cuda:
        raise RuntimeError("coat_b200: fp8matmul needs CUDA tensors (no CPU path exists)")
    if b.stride(0) != 1 or b.stride(1) != b.shape[0]:
        raise RuntimeError("fp8matmul: B must be the transposed view of a contiguous [N, K] matrix (K contiguous)")
    M, K = a.shape
    _, N = b.shape
    dev = a.device
    if output_quantize:
        c = torch.empty((M, N), device=dev, dtype=a.dtype)
        scale_c = torch.empty((M, N // QB), device=dev, dtype=torch.bfloat16)
    else:
        c = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
        scale_c = None
    if scale_a.dtype != scale_b.dtype:
        scale_b = scale_b.to(scale_a.dtype)
    with torch.cuda.device(dev):
        _call("coat_fp8_gemm", a.data_ptr(), b.data_ptr(), c.data_ptr(), None if scale_c is None else scale_c.data_ptr(),
              scale_a.data_ptr(), scale_b.data_ptr(), None if bias is None else bias.data_ptr(), M, N, K,
              _lib.fp8_enum_of(a), _lib.fp8_enum_of(b), _lib.float_dtype(scale_a),
              _lib.BF16 if bias is None else _lib.float_dtype(bias), int(bool(output_quantize)), QB if QB else 16,
              _flags(flags), _lib.stream_ptr(dev))
    if batched:
        c = c.reshape(BS, -1, N)
        if output_quantize:
            return c, scale_c.reshape(BS, -1, N // QB)
    elif output_quantize:
        return c, scale_c
    return c


def fp8_linear_forward(x, s, w, s_w, output_quantize, QB, bias=None):
    assert s.numel() == 1, f"X uses per-tensor quantization in linear forward, but the scale shape is {s.shape}"
    assert s_w.numel() == 1, f"W uses per-tensor quantization in linear forward, but the scale shape is {s_w.shape}"
    return fp8matmul(x, w.t(), output_quantize, s, s_w, QB, bias)


def fp8_linear_backward(x_t, s, g, s_g, g_t, w_t, s_w, QB, bias=None, stochastic=False, dgrad_quantize=False):
    assert s.numel() == 1, f"X uses per-tensor quantization in linear backward, but the scale shape is {s.shape}"
    assert s_g.numel() == 1, f"G uses per-tensor quantization in linear backward, but the scale shape is {s.shape}"
    assert s_w.numel() == 1, f"W uses per-tensor quantization in linear backward, but the scale shape is {s_w.shape}"
    batched = g.dim() == 3
    if batched:
        BS = g.shape[0]
        g = g.reshape(-1, g.shape[-1])
    if dgrad_quantize:
        y, s_y = fp8matmul(g, w_t.t(), True, s_g, s_w, QB, stochastic=stochastic)
    else:
        y = fp8matmul(g, w_t.t(), False, s_g, s_w, QB)
    w_g = fp8matmul(g_t, x_t.t(), False, s_g, s, QB)
    if batched:
        y = y.reshape(BS, -1, y.shape[-1])
        if dgrad_quantize and s_y.numel() > 1:
            s_y = s_y.reshape(BS, -1, s_y.shape[-1])
    if dgrad_quantize:
        return y, s_y, w_g
    return y, w_g
