"""GPU tests of the block-scaled (DeepSeek-style) path: the tcgen05 block-scaled GEMM against exact fp64
arithmetic on the same codes and scales, and the FP8DeepSeekLinear layer against an unquantised linear.
Tolerance of the GEMM: the result is bf16 of an fp32 accumulation: |err| <= 2^-7 |y| + 2^-7 rms(y)."""
import pytest
import torch

from coat_b200 import _lib
from coat_b200.activation.deepseek import FP8DeepSeekLinear, gemm_fp8_fp8_bf16_nt
from coat_b200.activation.real_quantization import fp8_quantize_perblock, fp8_quantize_transpose
from oracle import gemm as OG

pytestmark = pytest.mark.gpu


def operands(M, N, K, fmt_a=torch.float8_e4m3fn, seed=5):
    gen = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, K, generator=gen) * (1 + 10 * torch.rand(M, 1, generator=gen))).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    (qx, sx), _ = fp8_quantize_transpose(x, 128, fmt_a, scale_dtype=torch.float32)
    qw, sw = fp8_quantize_perblock(w, 128, torch.float8_e4m3fn, scale_dtype=torch.float32)
    return qx, sx.t().contiguous().t(), qw, sw


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 384, 512), (1024, 256, 1152), (384, 1280, 4096), (4096, 512, 256)])
@pytest.mark.parametrize("fmt_a", [torch.float8_e4m3fn, torch.float8_e5m2])
def test_blockscaled_gemm_against_exact_arithmetic(M, N, K, fmt_a):
    qx, sx, qw, sw = operands(M, N, K, fmt_a)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm_fp8_fp8_bf16_nt((qx, sx), (qw, sw), out)
    torch.cuda.synchronize()
    assert _lib.lib().coat_fp8_gemm_device_status() == 0
    ref = OG.blockscaled_matmul_fp64(qx.cpu(), sx.cpu(), qw.cpu(), sw.cpu())
    assert bool(OG.within_tolerance(out.cpu(), ref).all())


def test_blockscaled_gemm_many_tiles_and_ragged_rows():
    """More tiles than SMs (persistent loop, barrier phases across tiles) and a row count that is not a multiple
    of 128 (rows beyond M are neither scaled nor stored); checker computed in fp64 on the GPU."""
    M, N, K = 2000, 2560, 384
    gen = torch.Generator().manual_seed(6)
    qx = (torch.randn(M, K, generator=gen) * 40).to(torch.float8_e4m3fn).cuda()
    sx = (torch.rand(M, K // 128, generator=gen) * 0.05 + 0.001).cuda().t().contiguous().t()
    qw = (torch.randn(N, K, generator=gen) * 40).to(torch.float8_e4m3fn).cuda()
    sw = (torch.rand(N // 128, K // 128, generator=gen) * 0.02 + 0.001).cuda()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm_fp8_fp8_bf16_nt((qx, sx), (qw, sw), out)
    torch.cuda.synchronize()
    assert _lib.lib().coat_fp8_gemm_device_status() == 0
    ref = OG.blockscaled_matmul_fp64(qx, sx, qw, sw)
    assert bool(OG.within_tolerance(out, ref).all())


def test_blockscaled_gemm_scales_are_applied_per_k_block():
    """One K block scaled by 1000: the result must follow (a kernel that scaled per tile would not)."""
    M, N, K = 128, 128, 512
    qx, sx, qw, sw = operands(M, N, K)
    sx = sx.clone()
    sx[:, 2] *= 1000.0
    sx = sx.t().contiguous().t()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm_fp8_fp8_bf16_nt((qx, sx), (qw, sw), out)
    ref = OG.blockscaled_matmul_fp64(qx.cpu(), sx.cpu(), qw.cpu(), sw.cpu())
    assert bool(OG.within_tolerance(out.cpu(), ref).all())


def test_blockscaled_gemm_rejects_partial_blocks():
    qx, sx, qw, sw = operands(128, 128, 256)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.lib().coat_fp8_gemm_blockscaled(qx.data_ptr(), sx.data_ptr(), 128, qw.data_ptr(), sw.data_ptr(),
                                                        qx.data_ptr(), 128, 128, 200, 0, 0, None), "blockscaled")


def test_deepseek_linear_forward_backward_close_to_unquantised():
    """E4M3 everywhere (the reference's defaults): rounding leaves ~2.6 % rms per factor; outputs and gradients
    of one layer must agree with the bf16 layer to 6 % relative Frobenius error and cosine 0.997."""
    gen = torch.Generator().manual_seed(9)
    layer = FP8DeepSeekLinear(512, 768, bias=True).cuda().to(torch.bfloat16).train()
    with torch.no_grad():
        layer.weight.copy_(torch.randn(768, 512, generator=gen) * 0.03)
        layer.bias.zero_()
    x = torch.randn(4, 128, 512, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    up = (torch.randn(4, 128, 768, generator=gen) * 0.1).to(torch.bfloat16).cuda()
    y = layer(x)
    y.backward(up)
    xr = x.detach().float().requires_grad_(True)
    wr = layer.weight.detach().float().requires_grad_(True)
    yr = xr @ wr.t()
    yr.backward(up.float())

    def close(t, r, what):
        t, r = t.detach().double().flatten(), r.detach().double().flatten()
        rel = float((t - r).norm() / r.norm())
        cos = float(torch.dot(t, r) / (t.norm() * r.norm()))
        assert rel <= 0.06 and cos >= 0.997, f"{what}: relative error {rel:.4f}, cosine {cos:.5f}"

    close(y, yr, "output")
    close(x.grad, xr.grad, "input gradient")
    close(layer.weight.grad, wr.grad, "weight gradient")
    assert torch.allclose(layer.bias.grad.float(), up.float().sum((0, 1)), rtol=2e-2, atol=1e-2)
    layer.eval()
    with torch.no_grad():
        assert torch.equal(layer(x.detach()), torch.nn.functional.linear(x.detach(), layer.weight, layer.bias))
