"""CPU / fp64 restatement of the reference's FP8 matmul (TEST INFRASTRUCTURE ONLY).

coat/activation/real_quantization/linear.py:104-169 accumulates the FP8 products in fp32, multiplies by
float(scale_a) * float(scale_b), adds the bias and rounds to bf16 (or quantises 1xQB).  The order of the
fp32 accumulation is an implementation detail of the tensor-core kernel, so the checker computes the
products exactly (fp64 matmul of the decoded codes, as the reference's own test does with a torch matmul,
tests/test_fp8_linear.py:120-124) and the tests allow one bf16 ulp plus accumulation slack:
|err| <= 2^-7 |y| + 2^-7 rms(y)."""
import torch


def fp8_matmul_fp64(a, b_nk, scale_a, scale_b, bias=None):
    """a [M,K], b_nk [N,K] fp8 tensors -> fp64 [M,N]."""
    y = a.to(torch.float32).double() @ b_nk.to(torch.float32).double().t()
    y = y * (scale_a.float() * scale_b.float()).double()
    if bias is not None:
        y = y + bias.double()
    return y


def within_tolerance(c, ref):
    err = (c.double() - ref).abs()
    tol = 2.0 ** -7 * ref.abs() + 2.0 ** -7 * ref.pow(2).mean().sqrt()
    return err <= tol


def blockscaled_matmul_fp64(a, sa, b, sb):
    """a [M,K], b [N,K] fp8; sa [M, K/128], sb [N/128, K/128] fp32 -> fp64 [M,N]: every 1x128 segment of a and
    128x128 block of b dequantised exactly, products summed exactly (what deep_gemm.gemm_fp8_fp8_bf16_nt computes
    up to its fp32 accumulation order, coat/activation/deepseek/linear.py:10-16)."""
    M, K = a.shape
    N = b.shape[0]
    ad = a.to(torch.float32).double().reshape(M, K // 128, 128) * sa.double()[:, :, None]
    bd = b.to(torch.float32).double().reshape(N // 128, 128, K // 128, 128) * sb.double()[:, None, :, None]
    return ad.reshape(M, K) @ bd.reshape(N, K).t()
