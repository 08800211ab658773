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


def _nt(lhs, rhs):
    """out[M, N] = lhs[M, K] @ rhs[N, K]^T for (codes, scales) pairs in the layouts deepseek_check_stride asks for."""
    deepseek_check_stride(lhs, rhs)
    out = torch.empty((lhs[0].shape[0], rhs[0].shape[0]), device=lhs[0].device, dtype=torch.bfloat16)
    return gemm_fp8_fp8_bf16_nt(lhs, rhs, out)


def fp8_deepseek_linear_forward(x, s, w, s_w, QB, bias=None):
    """x [tokens, in] with 1x128 scales, w [out, in] with 128x128 scales -> [tokens, out].  `QB` and `bias` are
    accepted and ignored, as in the reference."""
    return _nt((x, s), (w, s_w))


def fp8_deepseek_linear_backward(x_t, s_t, g, s_g, g_t, s_g_t, w_t, s_w_t):
    """dgrad = g [tokens, out] @ w_t [in, out]^T; wgrad comes out transposed ([in, out] = x_t [in, tokens] @
    g_t [out, tokens]^T) and is turned round, as in the reference."""
    d_input = _nt((g, s_g), (w_t, s_w_t))
    d_weight_t = _nt((x_t, s_t), (g_t, s_g_t))
    return d_input, d_weight_t.t().contiguous()
