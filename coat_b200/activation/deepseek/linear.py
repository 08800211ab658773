"""Block-scaled linear forward / backward with the names and arguments of coat/activation/deepseek/linear.py:10-36.
Where the reference calls deep_gemm.gemm_fp8_fp8_bf16_nt, this calls the tcgen05 block-scaled GEMM behind the C ABI
(`gemm_fp8_fp8_bf16_nt` below has deep_gemm's calling convention)."""
import torch

from ... import _lib
from ..real_quantization._ops import _call


def deepseek_check_stride(x_fp8, y_fp8):
    assert x_fp8[0].stride(1) == 1
    assert x_fp8[1].stride(0) == 1
    assert y_fp8[0].stride(1) == 1
    assert y_fp8[1].stride(1) == 1


def gemm_fp8_fp8_bf16_nt(lhs, rhs, out):
    """lhs = (A [M,K] fp8, scales [M, K/128] fp32 with stride(0) == 1), rhs = (B [N,K] fp8, scales [N/128, K/128]
    fp32 contiguous), out [M,N] bf16:  out = (A * scales_a) @ (B * scales_b)^T with fp32 accumulation."""
    (a, sa), (b, sb) = lhs, rhs
    if not a.is_cuda:
        raise RuntimeError("coat_b200: the block-scaled GEMM needs CUDA tensors (no CPU path exists)")
    M, K = a.shape
    N = b.shape[0]
    assert b.shape[1] == K and out.shape == (M, N) and out.dtype == torch.bfloat16 and out.is_contiguous()
    assert a.stride(1) == 1 and a.stride(0) == K and b.stride(1) == 1 and b.stride(0) == K
    assert sa.dtype == torch.float32 and sb.dtype == torch.float32
    assert sa.shape == (M, K // 128) and sa.stride(0) == 1 and sb.shape == (N // 128, K // 128) and sb.is_contiguous()
    lds_a = sa.stride(1) if sa.shape[1] > 1 else M
    with torch.cuda.device(a.device):
        _call("coat_fp8_gemm_blockscaled", a.data_ptr(), sa.data_ptr(), lds_a, b.data_ptr(), sb.data_ptr(),
              out.data_ptr(), M, N, K, _lib.fp8_enum_of(a), _lib.fp8_enum_of(b), _lib.stream_ptr(a.device))
    return out


def fp8_deepseek_linear_forward(x, s, w, s_w, QB, bias=None):
    x_fp8, w_fp8 = (x, s), (w, s_w)
    out = torch.empty((x.shape[0], w.shape[0]), device=x.device, dtype=torch.bfloat16)
    deepseek_check_stride(x_fp8, w_fp8)
    gemm_fp8_fp8_bf16_nt(x_fp8, w_fp8, out)
    return out


def fp8_deepseek_linear_backward(x_t, s_t, g, s_g, g_t, s_g_t, w_t, s_w_t):
    # dgrad
    g_fp8, w_t_fp8 = (g, s_g), (w_t, s_w_t)
    y = torch.empty((g.shape[0], w_t.shape[0]), device=x_t.device, dtype=torch.bfloat16)
    deepseek_check_stride(g_fp8, w_t_fp8)
    gemm_fp8_fp8_bf16_nt(g_fp8, w_t_fp8, y)
    # wgrad, produced transposed ([in, out]) as in the reference and turned round at the end
    x_t_fp8, g_t_fp8 = (x_t, s_t), (g_t, s_g_t)
    w_g_t = torch.empty((x_t.shape[0], g_t.shape[0]), device=x_t.device, dtype=torch.bfloat16)
    deepseek_check_stride(x_t_fp8, g_t_fp8)
    gemm_fp8_fp8_bf16_nt(x_t_fp8, g_t_fp8, w_g_t)
    return y, w_g_t.t().contiguous()
