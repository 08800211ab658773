"""GPU parity tests of the tcgen05 FP8 GEMM through the reference-shaped wrappers (fp8matmul,
fp8_linear_forward / backward, FP8Linear).  Tolerance fixed up front: against an fp64 matmul of the same
FP8 codes, |err| <= 2^-7 |y| + 2^-7 rms(y) (one bf16 ulp plus fp32 accumulation-order slack)."""
import pytest
import torch

from oracle import gemm as G
from oracle import quant as Q

pytestmark = pytest.mark.gpu


def mods():
    from coat_b200 import _lib
    from coat_b200.activation.real_quantization import linear
    return linear, _lib


def codes(rows, cols, seed, dtype, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    return Q.cast_fp8(torch.randn(rows, cols, generator=gen) * scale, dtype)


def sc(v):
    return torch.tensor(v, dtype=torch.bfloat16, device="cuda")


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 512, 1024), (200, 300, 272), (16, 48, 4096), (384, 256, 144)])
@pytest.mark.parametrize("fa,fb", [(torch.float8_e4m3fn, torch.float8_e4m3fn), (torch.float8_e5m2, torch.float8_e4m3fn)])
def test_matmul_against_fp64(M, N, K, fa, fb):
    linear, _lib = mods()
    a, b = codes(M, K, 1, fa, 30.0), codes(N, K, 2, fb, 1.0)
    sa, sb = sc(0.0123), sc(0.5)
    c = linear.fp8matmul(a.cuda(), b.cuda().t(), False, sa, sb, 16)
    assert c.dtype == torch.bfloat16 and c.shape == (M, N)
    ref = G.fp8_matmul_fp64(a, b, sa.cpu(), sb.cpu())
    assert G.within_tolerance(c.cpu(), ref).all()
    assert _lib.lib().coat_fp8_gemm_device_status() == 0


def test_bias_batched_and_contiguity_rule():
    linear, _lib = mods()
    a, b = codes(6 * 40, 256, 3, torch.float8_e4m3fn), codes(320, 256, 4, torch.float8_e4m3fn)
    bias = torch.linspace(-2, 2, 320).to(torch.bfloat16)
    sa, sb = sc(0.02), sc(0.03)
    c = linear.fp8matmul(a.reshape(6, 40, 256).cuda(), b.cuda().t(), False, sa, sb, 16, bias.cuda())
    assert c.shape == (6, 40, 320)
    ref = G.fp8_matmul_fp64(a, b, sa.cpu(), sb.cpu(), bias.float())
    assert G.within_tolerance(c.reshape(-1, 320).cpu(), ref).all()
    with pytest.raises(RuntimeError, match="contiguous"):
        linear.fp8matmul(a.cuda(), b.cuda().t().contiguous(), False, sa, sb, 16)   # N contiguous: not accepted


def test_fused_output_quantisation():
    """1x16 quantisation of the result inside the epilogue (linear.py:139-164): scales and codes against a
    quantisation of the fp64 result; equal nearly everywhere, never more than one code step apart."""
    linear, _lib = mods()
    M, N, K = 256, 512, 384
    a, b = codes(M, K, 5, torch.float8_e4m3fn, 20.0), codes(N, K, 6, torch.float8_e4m3fn)
    sa, sb = sc(0.01), sc(0.25)
    c, s_c = linear.fp8matmul(a.cuda(), b.cuda().t(), True, sa, sb, 16)
    assert c.dtype == torch.float8_e4m3fn and s_c.dtype == torch.bfloat16 and s_c.shape == (M, N // 16)
    ref = G.fp8_matmul_fp64(a, b, sa.cpu(), sb.cpu()).float()
    eq, es = Q.fp8_quantize(ref, 16, "E4M3")
    assert (s_c.cpu().view(torch.int16) == es.view(torch.int16)).float().mean() >= 0.99
    cu, eu = c.cpu().view(torch.uint8).to(torch.int16), eq.view(torch.uint8).to(torch.int16)
    assert (cu == eu).float().mean() >= 0.98 and (cu - eu).abs().max() <= 1
    deq = Q.fp8_dequantize(c.cpu(), s_c.cpu(), 16).float()
    assert ((deq - ref).abs() <= 0.07 * ref.abs() + ref.abs().max() * 2 ** -9).all()


def test_linear_forward_backward_wrappers():
    linear, _lib = mods()
    import coat_b200.activation.real_quantization as r
    T, H, O = 512, 256, 384
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(T, H, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(O, H, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    g = (torch.randn(T, O, generator=gen) * 1e-2).to(torch.bfloat16).cuda()
    qx, sx, qx_t = r.fp8_quantize_pertensor_transpose(x, 16, "E4M3", transpose_output_2d=True)
    qw, sw, qw_t = r.fp8_quantize_pertensor_transpose(w, 16, "E4M3", transpose_output_2d=True)
    qg, sg, qg_t = r.fp8_quantize_pertensor_transpose(g, 16, "E5M2", transpose_output_2d=True)
    y = linear.fp8_linear_forward(qx, sx, qw, sw, False, 0)
    assert G.within_tolerance(y.cpu(), G.fp8_matmul_fp64(qx.cpu(), qw.cpu(), sx.cpu(), sw.cpu())).all()
    dx, dw = linear.fp8_linear_backward(qx_t, sx, qg, sg, qg_t, qw_t, sw, 16)
    assert dx.shape == (T, H) and dw.shape == (O, H)
    assert G.within_tolerance(dx.cpu(), G.fp8_matmul_fp64(qg.cpu(), qw_t.cpu(), sg.cpu(), sw.cpu())).all()
    assert G.within_tolerance(dw.cpu(), G.fp8_matmul_fp64(qg_t.cpu(), qx_t.cpu(), sg.cpu(), sx.cpu())).all()
    # and against the unquantised bf16 linear: FP8 quantisation noise only
    rel = lambda p, q: ((p.float() - q.float()).norm() / q.float().norm()).item()
    assert rel(y, x @ w.t()) < 0.06 and rel(dx, g @ w) < 0.12 and rel(dw, g.t() @ x) < 0.12


def test_fp8linear_module_trains():
    from coat_b200.activation.real_quantization.fp8linear import FP8Linear
    torch.manual_seed(0)
    lin = FP8Linear(256, 384, bias=True, device="cuda").to(torch.bfloat16).train()
    ref = torch.nn.Linear(256, 384, bias=True, device="cuda").to(torch.bfloat16)
    ref.load_state_dict(lin.state_dict())
    x = torch.randn(4, 128, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    x2 = x.detach().clone().requires_grad_(True)
    y, y2 = lin(x), ref(x2)
    gy = torch.randn_like(y) * 1e-2
    y.backward(gy)
    y2.backward(gy)
    rel = lambda p, q: ((p.float() - q.float()).norm() / q.float().norm()).item()
    assert rel(y, y2) < 0.06 and rel(x.grad, x2.grad) < 0.12 and rel(lin.weight.grad, ref.weight.grad) < 0.12
    assert torch.allclose(lin.bias.grad.float(), ref.bias.grad.float(), rtol=2e-2, atol=1e-3)
    lin.eval()
    assert torch.equal(lin(x.detach()), ref(x.detach()))


def test_llama_mlp_shapes_sampled():
    """The FP8 linear benchmark configuration at full size (8192 x 4096 x 11008, forward, dgrad with E5M2 gradients,
    wgrad); checked on 64 sampled rows against the fp64 product."""
    linear, _lib = mods()
    M, H, I = 8192, 4096, 11008
    gen = torch.Generator(device="cuda").manual_seed(2)
    x = Q.cast_fp8(torch.randn(M, H, generator=gen, device="cuda") * 50, torch.float8_e4m3fn)
    w = Q.cast_fp8(torch.randn(I, H, generator=gen, device="cuda") * 50, torch.float8_e4m3fn)
    g = Q.cast_fp8(torch.randn(M, I, generator=gen, device="cuda") * 500, torch.float8_e5m2)
    sx, sw, sg = sc(0.02), sc(0.0004), sc(2e-5)
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(0))[:64].cuda()

    def check(c, a, b_nk, s1, s2, pick):
        ref = G.fp8_matmul_fp64(a[pick], b_nk, s1, s2)
        assert G.within_tolerance(c[pick], ref).all()

    y = linear.fp8_linear_forward(x, sx, w, sw, False, 0)
    check(y, x, w, sx, sw, rows)
    w_t = w.view(torch.uint8).t().contiguous().view(w.dtype)
    x_t = x.view(torch.uint8).t().contiguous().view(x.dtype)
    g_t = g.view(torch.uint8).t().contiguous().view(g.dtype)
    dx, dw = linear.fp8_linear_backward(x_t, sx, g, sg, g_t, w_t, sw, 16)
    check(dx, g, w_t, sg, sw, rows)
    check(dw, g_t, x_t, sg, sx, rows[:32] % I)
    assert _lib.lib().coat_fp8_gemm_device_status() == 0


@pytest.mark.parametrize("M,N,K,quantize", [
    (2112, 5200, 512, False),     # CTA pairs (K < 6144): 9 x 21 pair tiles on 74 pairs, ragged in M and N, several rounds
    (4000, 2832, 6272, False),    # 256-row tiles (K >= 6144): 16 x 12 tiles on 148 SMs, a split last round, ragged edges
    (128, 40192, 256, False),     # 128-row tiles (M <= 128): 157 tiles, two rounds
    (1536, 4096, 384, True),      # quantising epilogue over several rounds of the pair kernel
])
def test_many_tiles_per_sm(M, N, K, quantize):
    """More tiles than SMs, so that the persistent loops, the barrier phases across tiles and the tile walks of all
    three kernels are exercised; checked against an fp64 GEMM of the same codes computed on the GPU."""
    linear, _lib = mods()
    a, b = codes(M, K, 11, torch.float8_e4m3fn, 20.0).cuda(), codes(N, K, 12, torch.float8_e4m3fn, 1.0).cuda()
    sa, sb = sc(0.01), sc(0.25)
    ref = G.fp8_matmul_fp64(a, b, sa, sb)
    if not quantize:
        c = linear.fp8matmul(a, b.t(), False, sa, sb, 16)
        assert bool(G.within_tolerance(c, ref).all())
    else:
        q, s = linear.fp8matmul(a, b.t(), True, sa, sb, 16)
        deq = (q.float().reshape(M, N // 16, 16) * s.float().unsqueeze(-1)).reshape(M, N).double()
        # one E4M3 rounding of a value scaled into [0, 448]: half a step of 2^-3 relative, plus the bf16 scale
        assert bool(((deq - ref).abs() <= 0.07 * ref.abs().reshape(M, N // 16, 16).amax(-1, keepdim=True)
                     .expand(-1, -1, 16).reshape(M, N) + 1e-6).all())
    torch.cuda.synchronize()
    assert _lib.lib().coat_fp8_gemm_device_status() == 0
