"""GPU parity tests of the fused quantize-on-save operators against the torch restatement
(oracle/fused.py), through the python mirror of the reference API.

Operators without a transcendental (gated product, residual add) must agree BIT FOR BIT under IEEE
division.  SiLU / GELU evaluate exp / erf with libdevice on the GPU and libm on the CPU (last-place
differences), and RMSNorm sums in a different order, so those are held to the tolerances written in
each test.  The same operators are compared with the reference's own Triton kernels, in the default mode and at
the benchmark shapes, in test_vs_reference_triton_gpu.py."""
import pytest
import torch

from oracle import fused as F
from oracle import quant as Q

pytestmark = pytest.mark.gpu
IEEE = 1
QB = 16


def R():
    import coat_b200.activation.real_quantization as r
    return r


def qinput(M, N, seed, scale=1.0, fmt="E4M3"):
    gen = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, N, generator=gen) * scale).to(torch.bfloat16)
    return Q.fp8_quantize(x, QB, fmt)


def grad(M, N, seed):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(M, N, generator=gen) * 1e-2).to(torch.bfloat16)


def frac_equal(a, b):
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    view = {1: torch.uint8, 2: torch.int16, 4: torch.int32}[a.element_size()]
    return (a.view(view) == b.view(view)).float().mean().item()


def bf16_ulps(a, b):
    """|a-b| in units of the bf16 spacing at |b| (inputs bf16)."""
    a, b = a.detach().cpu().float(), b.detach().cpu().float()
    ulp = torch.exp2(torch.floor(torch.log2(torch.maximum(b.abs(), torch.tensor(1e-30)))) - 7)
    return ((a - b).abs() / ulp)


def code_steps(a, b):
    """Distance in code steps between two fp8 tensors of equal sign pattern (sign-magnitude codes)."""
    a, b = a.detach().cpu().view(torch.uint8).to(torch.int16), b.detach().cpu().view(torch.uint8).to(torch.int16)
    return (a - b).abs()


def same(a, b):
    assert frac_equal(a, b) == 1.0


def test_silu_forward():
    r = R()
    q, s = qinput(256, 512, 1, scale=2.0)
    y, s_y = r.fp8_silu_forward(q.cuda(), s.cuda(), QB, flags=IEEE)
    ey, es = F.silu_forward(q, s, QB)
    assert y.dtype == q.dtype and s_y.dtype == s.dtype
    assert frac_equal(s_y, es) >= 0.999
    assert frac_equal(y, ey) >= 0.999 and code_steps(y, ey).max() <= 1
    y3, s3 = r.fp8_silu_forward(q.reshape(4, 64, 512).cuda(), s.reshape(4, 64, 32).cuda(), QB, flags=IEEE)
    assert y3.shape == (4, 64, 512) and s3.shape == (4, 64, 32) and torch.equal(y3.reshape(256, 512).view(torch.uint8), y.view(torch.uint8))


@pytest.mark.parametrize("gelu", [False, True])
def test_activation_backward(gelu):
    r = R()
    q, s = qinput(256, 512, 2, scale=2.0)
    g = grad(256, 512, 3)
    value = (F.gelu_backward_value if gelu else F.silu_backward_value)(q, s, g, QB)
    ey, es_y, es_max, eq, eq_t = F.per_tensor_from_value(value, QB, "E5M2")
    if gelu:
        qy, s_max = r.fp8_gelu_backward(q.cuda(), s.cuda(), g.cuda(), QB, "E5M2", flags=IEEE)
    else:
        y, s_y = r.fp8_silu_backward(q.cuda(), s.cuda(), g.cuda(), QB, "E5M2", flags=IEEE)
        assert y.dtype == torch.bfloat16 and s_y.dtype == torch.bfloat16
        # bf16 result: at most one bf16 step from the restatement, identical nearly everywhere
        assert bf16_ulps(y, ey).max() <= 1.01 and frac_equal(y, ey) >= 0.995
        assert frac_equal(s_y, es_y) >= 0.995
        qy, s_max, qy_t = r.fp8_silu_backward(q.cuda(), s.cuda(), g.cuda(), QB, "E5M2", output_quantized_transpose=True,
                                              flags=IEEE)
        assert torch.equal(qy.view(torch.uint8).t(), qy_t.view(torch.uint8))
    assert qy.dtype == torch.float8_e5m2
    assert abs(s_max.float().item() - es_max.float().item()) <= es_max.float().item() * 2 ** -7
    if s_max.float().item() == es_max.float().item():
        assert frac_equal(qy, eq) >= (0.98 if gelu else 0.995) and code_steps(qy, eq).max() <= 1


def test_gelu_forward():
    r = R()
    q, s = qinput(128, 256, 4, scale=2.0)
    value = F.gelu_forward_value(q, s, QB)
    ey, es_y, es_max, eq, eq_t = F.per_tensor_from_value(value, QB, "E4M3")
    qy, s_max, qy_t = r.fp8_gelu_forward(q.cuda(), s.cuda(), QB, flags=IEEE)
    assert torch.equal(qy.view(torch.uint8).t(), qy_t.view(torch.uint8))
    assert abs(s_max.float().item() - es_max.float().item()) <= es_max.float().item() * 2 ** -7
    if s_max.float().item() == es_max.float().item():
        assert frac_equal(qy, eq) >= 0.98 and code_steps(qy, eq).max() <= 1


def test_mul_forward_bit_exact():
    r = R()
    q1, s1 = qinput(256, 384, 5)
    q2, s2 = qinput(256, 384, 6, scale=3.0)
    ey, es_y, es_max, eq, eq_t = F.per_tensor_from_value(F.mul_forward_value(q1, s1, q2, s2, QB), QB, "E4M3")
    qy, s_max, qy_t = r.fp8_mul_forward(q1.cuda(), s1.cuda(), q2.cuda(), s2.cuda(), QB, flags=IEEE)
    same(s_max, es_max)
    same(qy, eq)
    same(qy_t, eq_t)
    q3, _, q3_t = r.fp8_mul_forward(q1.reshape(2, 128, 384).cuda(), s1.reshape(2, 128, 24).cuda(),
                                    q2.reshape(2, 128, 384).cuda(), s2.reshape(2, 128, 24).cuda(), QB,
                                    transpose_output_2d=True, flags=IEEE)
    assert q3.shape == (2, 128, 384) and q3_t.shape == (384, 256)


def test_mul_backward_bit_exact():
    r = R()
    q1, s1 = qinput(128, 256, 7)
    q2, s2 = qinput(128, 256, 8)
    g = grad(128, 256, 9)
    v1, v2 = F.mul_backward_values(q1, s1, q2, s2, g, QB)
    y1, (y2, s_y2) = r.fp8_mul_backward(q1.cuda(), s1.cuda(), q2.cuda(), s2.cuda(), g.cuda(), QB, "E5M2", flags=IEEE)
    same(y1, v1.to(torch.bfloat16))
    same(y2, v2.to(torch.bfloat16))
    same(s_y2, Q.group_scales(v2, QB, "E5M2").to(torch.bfloat16))
    ey, es_y, es_max, eq, eq_t = F.per_tensor_from_value(v2, QB, "E5M2")
    y1b, (qy2, s_max, qy2_t) = r.fp8_mul_backward(q1.cuda(), s1.cuda(), q2.cuda(), s2.cuda(), g.cuda(), QB, "E5M2",
                                                  output_quantized_transpose=True, flags=IEEE)
    same(y1b, y1)
    same(s_max, es_max)
    same(qy2, eq)
    same(qy2_t, eq_t)


def test_add_bit_exact():
    r = R()
    gen = torch.Generator().manual_seed(10)
    a = torch.randn(192, 256, generator=gen).to(torch.bfloat16)
    b = (torch.randn(192, 256, generator=gen) * 0.3).to(torch.bfloat16)
    y1, (y2, s_y2) = r.fp8_add_Ifp_Ifp_Ofp_Og16(a.cuda(), b.cuda(), torch.float8_e4m3fn, QB, flags=IEEE)
    e1, (e2, es2) = F.add_forward(a, b, "E4M3", QB)
    same(y1, e1)
    same(y2, e2)
    same(s_y2, es2)
    # backward flavour: bf16 sum, per-tensor E5M2 of the bf16 sum, group scales; fp32 first operand
    v = a.float() + b.float()
    ey, es_y, es_max, eq, _ = F.per_tensor_from_value(v, QB, "E5M2", transposed=False)
    y1, (qy2, s_max, s_y2) = r.fp8_add_Ifp_Ifp_Ofp_Opt(a.float().cuda(), b.cuda(), QB, "E5M2", flags=IEEE)
    same(y1, ey)
    same(s_y2, es_y)
    same(s_max, es_max)
    same(qy2, eq)


@pytest.mark.parametrize("N", [512, 2048, 4096, 5120, 10240])   # 1, 2 and 4 segments per thread
def test_rmsnorm_forward_backward(N):
    r = R()
    M = 64
    q, s = qinput(M, N, 11)
    gen = torch.Generator().manual_seed(12)
    w = (1 + 0.1 * torch.randn(N, generator=gen)).to(torch.bfloat16)
    value, erstd = F.rmsnorm_forward_value(q, s, w, QB, 1e-5)
    ey, _, _, _, _ = F.per_tensor_from_value(value, QB, "E4M3")
    es_max = F.rmsnorm_row_scales(value, "E4M3").max()
    eq = Q.fp8_division(ey, "E4M3", es_max)
    qy, s_max, qy_t, (w_ctx, rstd, nw) = r.fp8_rmsnorm_forward(q.cuda(), s.cuda(), w.cuda(), QB, 1e-5, flags=IEEE)
    # rstd: different summation order and an approximate sqrt: 4 fp32 ulps
    assert torch.allclose(rstd.cpu(), erstd, rtol=5e-7, atol=0)
    assert torch.equal(qy.view(torch.uint8).t(), qy_t.view(torch.uint8))
    assert abs(s_max.float().item() - es_max.float().item()) <= es_max.float().item() * 2 ** -7
    if s_max.float().item() == es_max.float().item():
        assert frac_equal(qy, eq) >= 0.99 and code_steps(qy, eq).max() <= 1
    g = grad(M, N, 13)
    dx, dw = r.fp8_rmsnorm_backward(q.cuda(), s.cuda(), g.cuda(), w.cuda(), rstd, QB, nw)
    edx, edw = F.rmsnorm_backward(q, s, g, w, erstd, QB)
    assert dx.dtype == torch.bfloat16 and dw.dtype == w.dtype and dw.shape == (N,)
    assert frac_equal(dx, edx) >= 0.97 and (dx.cpu().float() - edx.float()).abs().max() <= 2 ** -7 * edx.float().abs().max()
    # the reference's own tolerance for the weight gradient (tests/test_fp8_norm.py:184)
    assert torch.allclose(dw.cpu().float(), edw, rtol=1e-2, atol=1e-3 * edw.abs().max().item())
    # deterministic: a second run gives the same bits (the reference's lock-ordered sum does not)
    dx2, dw2 = r.fp8_rmsnorm_backward(q.cuda(), s.cuda(), g.cuda(), w.cuda(), rstd, QB, nw)
    assert torch.equal(dw, dw2) and torch.equal(dx, dx2)


@pytest.mark.parametrize("N", [512, 4096, 5120])
@pytest.mark.parametrize("affine", [False, True])
def test_layernorm_forward_backward(N, affine):
    """LayerNorm without and with weight/bias against the oracle and against torch's layer_norm autograd on the
    dequantised input.  mean / rstd: summation order only (5e-7 relative resp. absolute on the mean's scale)."""
    r = R()
    M = 64
    q, s = qinput(M, N, 21)
    gen = torch.Generator().manual_seed(22)
    w = (1 + 0.1 * torch.randn(N, generator=gen)).to(torch.bfloat16) if affine else None
    b = (0.1 * torch.randn(N, generator=gen)).to(torch.bfloat16) if affine else None
    value, emean, erstd = F.layernorm_forward_value(q, s, w, b, QB, 1e-5)
    es_max = F.rmsnorm_row_scales(value, "E4M3").max()
    eq = Q.fp8_division(value, "E4M3", es_max)
    if affine:
        qy, s_max, qy_t, (w_ctx, b_ctx, mean, rstd, nw) = r.fp8_layernorm_param_forward(
            q.cuda(), s.cuda(), w.cuda(), b.cuda(), QB, 1e-5, flags=IEEE)
    else:
        qy, s_max, qy_t, (mean, rstd, nw) = r.fp8_layernorm_noparam_forward(q.cuda(), s.cuda(), QB, 1e-5, flags=IEEE)
    v = F.dequant(q, s, QB)
    assert torch.allclose(mean.cpu(), emean, rtol=0, atol=5e-7 * float(v.abs().max()))
    assert torch.allclose(rstd.cpu(), erstd, rtol=1e-6, atol=0)
    assert torch.equal(qy.view(torch.uint8).t(), qy_t.view(torch.uint8))
    assert abs(s_max.float().item() - es_max.float().item()) <= es_max.float().item() * 2 ** -7
    if s_max.float().item() == es_max.float().item():
        assert frac_equal(qy, eq) >= 0.99 and code_steps(qy, eq).max() <= 1
    g = grad(M, N, 23)
    if affine:
        dx, dw, db = r.fp8_layernorm_param_backward(q.cuda(), s.cuda(), g.cuda(), QB, w.cuda(), b.cuda(), mean, rstd, nw)
    else:
        dx = r.fp8_layernorm_noparam_backward(q.cuda(), s.cuda(), g.cuda(), QB, mean, rstd, nw)
    edx, edw, edb = F.layernorm_backward(q, s, g, w, emean, erstd, QB)
    assert dx.dtype == torch.bfloat16
    assert frac_equal(dx, edx) >= 0.97 and (dx.cpu().float() - edx.float()).abs().max() <= 2 ** -7 * edx.float().abs().max()
    # torch autograd of layer_norm on the dequantised input agrees with the oracle's formulas
    vv = v.clone().requires_grad_(True)
    ww = None if w is None else w.float().requires_grad_(True)
    bb = None if b is None else b.float().requires_grad_(True)
    torch.nn.functional.layer_norm(vv, (N,), ww, bb, 1e-5).backward(g.float())
    assert torch.allclose(edx.float(), vv.grad, rtol=2e-2, atol=2e-2 * float(vv.grad.abs().max()))
    if affine:
        assert dw.dtype == w.dtype and dw.shape == (N,) and db.shape == (N,)
        assert torch.allclose(dw.cpu().float(), edw, rtol=1e-2, atol=1e-3 * edw.abs().max().item())
        assert torch.allclose(db.cpu().float(), edb, rtol=1e-2, atol=1e-3 * edb.abs().max().item())
        assert torch.allclose(edw, ww.grad, rtol=1e-3, atol=1e-3 * float(ww.grad.abs().max()))
        assert torch.allclose(edb, bb.grad, rtol=1e-3, atol=1e-3 * float(bb.grad.abs().max()))
        dx2, dw2, db2 = r.fp8_layernorm_param_backward(q.cuda(), s.cuda(), g.cuda(), QB, w.cuda(), b.cuda(), mean, rstd, nw)
        assert torch.equal(dw, dw2) and torch.equal(db, db2) and torch.equal(dx, dx2)


def test_layernorm_batched_shapes_and_limits():
    r = R()
    q, s = qinput(64, 512, 24)
    q3, s3 = q.view(4, 16, 512).cuda(), s.view(4, 16, -1).cuda()
    qy, s_max, qy_t, (mean, rstd, nw) = r.fp8_layernorm_noparam_forward(q3, s3, QB, 1e-5)
    assert qy.shape == (4, 16, 512) and qy_t.shape == (4, 16, 512) and mean.shape == (64,)   # the reference reshapes the [N, M] copy to (BS, -1, N)
    qy2, _, qy_t2, _ = r.fp8_layernorm_noparam_forward(q3, s3, QB, 1e-5, transpose_output_2d=True)
    assert qy_t2.shape == (512, 64) and torch.equal(qy_t2.view(torch.uint8), qy.view(torch.uint8).view(64, 512).t())
    dx = r.fp8_layernorm_noparam_backward(q3, s3, grad(64, 512, 25).view(4, 16, 512).cuda(), QB, mean, rstd, nw)
    assert dx.shape == (4, 16, 512)
    with pytest.raises(NotImplementedError):
        r.fp8_layernorm_noparam_backward(q3, s3, dx, QB, mean, rstd, nw, stochastic=True)


@pytest.mark.parametrize("n_more", [1, 2])
def test_rmsnorm_backward_sums_its_upstream_gradients(n_more):
    """`more_g`: the kernel's bf16 left-to-right sum of the addends gives the bits of passing torch's `a + b (+ c)`."""
    import torch
    r = R()
    M, N = 96, 4096
    q, s = qinput(M, N, 41)
    w = (1 + 0.1 * torch.randn(N, generator=torch.Generator().manual_seed(42))).to(torch.bfloat16).cuda()
    q, s = q.cuda(), s.cuda()
    _, _, _, (_, rstd, nw) = r.fp8_rmsnorm_forward(q, s, w, QB, 1e-5)
    gs = [grad(M, N, 43 + i).cuda() for i in range(1 + n_more)]
    total = gs[0] + gs[1] if n_more == 1 else gs[0] + gs[1] + gs[2]
    dx_ref, dw_ref = r.fp8_rmsnorm_backward(q, s, total, w, rstd, QB, nw)
    dx, dw = r.fp8_rmsnorm_backward(q, s, gs[0], w, rstd, QB, nw, more_g=tuple(gs[1:]))
    assert torch.equal(dx, dx_ref) and torch.equal(dw, dw_ref)


@pytest.mark.parametrize("flags", [None, IEEE])
def test_mul_silu_backward_equals_the_two_operators(flags):
    """The one-kernel backward of silu(gate) * up gives, bit for bit, what fp8_mul_backward followed by
    fp8_silu_backward give (codes, transposed codes and per-tensor scales of both gradients)."""
    import torch
    r = R()
    M, N = 272, 1408
    silu_q, silu_s = qinput(M, N, 51)
    up_q, up_s = qinput(M, N, 52)
    gate_q, gate_s = qinput(M, N, 53, scale=2.0)
    g = grad(M, N, 54).cuda()
    args = [t.cuda() for t in (silu_q, silu_s, up_q, up_s)]
    gate_q, gate_s = gate_q.cuda(), gate_s.cuda()
    g1, (q_up, s_up, q_up_t) = r.fp8_mul_backward(*args, g, QB, "E5M2", output_quantized_transpose=True, flags=flags)
    q_gate, s_gate, q_gate_t = r.fp8_silu_backward(gate_q, gate_s, g1, QB, "E5M2", output_quantized_transpose=True,
                                                   flags=flags)
    (f_up, fs_up, f_up_t), (f_gate, fs_gate, f_gate_t) = r.fp8_mul_silu_backward(*args, gate_q, gate_s, g, QB, "E5M2",
                                                                                   flags=flags)
    u8 = lambda t: t.view(torch.uint8)
    assert fs_up == s_up and fs_gate == s_gate
    assert torch.equal(u8(f_up), u8(q_up)) and torch.equal(u8(f_up_t), u8(q_up_t))
    assert torch.equal(u8(f_gate), u8(q_gate)) and torch.equal(u8(f_gate_t), u8(q_gate_t))
    # batched input keeps the leading dimension on the straight codes
    b = lambda t: t.view(2, M // 2, -1)
    (b_up, _, b_up_t), _ = r.fp8_mul_silu_backward(b(args[0]), b(args[1]), b(args[2]), b(args[3]), b(gate_q), b(gate_s),
                                                   b(g), QB, "E5M2", flags=flags)
    assert b_up.shape == (2, M // 2, N) and torch.equal(u8(b_up).view(M, N), u8(q_up)) and b_up_t.shape == (N, M)


@pytest.mark.parametrize("flags", [None, IEEE])
def test_silu_mul_forward_equals_the_two_operators(flags):
    """The one-kernel forward of silu(gate) * up gives, bit for bit, what fp8_silu_forward followed by
    fp8_mul_forward give (the saved silu codes and scales, the product's codes, transposed codes and scale)."""
    import torch
    r = R()
    M, N = 272, 1408
    gate_q, gate_s = qinput(M, N, 61, scale=2.0)
    up_q, up_s = qinput(M, N, 62)
    gate_q, gate_s, up_q, up_s = (t.cuda() for t in (gate_q, gate_s, up_q, up_s))
    silu_q, silu_s = r.fp8_silu_forward(gate_q, gate_s, QB, flags=flags)
    mul_q, mul_s, mul_t = r.fp8_mul_forward(silu_q, silu_s, up_q, up_s, QB, transpose_output_2d=True, flags=flags)
    (f_silu_q, f_silu_s), (f_mul_q, f_mul_s, f_mul_t) = r.fp8_silu_mul_forward(gate_q, gate_s, up_q, up_s, QB,
                                                                               transpose_output_2d=True, flags=flags)
    u8 = lambda t: t.view(torch.uint8)
    assert torch.equal(u8(f_silu_q), u8(silu_q)) and torch.equal(f_silu_s, silu_s)
    assert f_mul_s == mul_s and torch.equal(u8(f_mul_q), u8(mul_q)) and torch.equal(u8(f_mul_t), u8(mul_t))


@pytest.mark.parametrize("M,N", [(256, 384), (1040, 1280), (4096, 11008)])
@pytest.mark.parametrize("flags", [0, IEEE])
def test_mul_forward_one_launch_equals_the_two_kernel_form(M, N, flags):
    """fp8_mul_forward as one cooperative launch (the product recomputed from the FP8 inputs in the second pass)
    against the two-kernel form (bf16 product in memory + division/transpose): same scale, codes and transposed
    codes, in both division modes; ragged tile edges (1040 rows = 8 tiles + 16 rows) included."""
    r = R()
    from coat_b200 import _lib
    from coat_b200.activation.real_quantization import _ops
    q1, s1 = qinput(M, N, 31)
    q2, s2 = qinput(M, N, 32, scale=3.0)
    args = (q1.cuda(), s1.cuda(), q2.cuda(), s2.cuda(), QB)
    assert _ops._ONE_LAUNCH
    one = r.fp8_mul_forward(*args, flags=flags)
    try:
        _ops._ONE_LAUNCH = False
        two = r.fp8_mul_forward(*args, flags=flags)
    finally:
        _ops._ONE_LAUNCH = True
    for a, b in zip(one, two):
        same(a, b)
    assert _lib.lib().coat_fp8_quantize_device_status() == 0
