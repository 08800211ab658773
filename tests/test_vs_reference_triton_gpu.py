"""GPU parity tests against the REFERENCE ITSELF: the reference's Triton kernels and python wrappers
(coat/activation/real_quantization/*.py, staged unmodified by oracle/build_ref.py into oracle/_ref/coat_ref/)
run on the same GPU, on the same tensors, next to this repository's CUDA kernels in their DEFAULT mode
(no IEEE-division flag: the mode a user gets).

Bar, stated up front:
  * every operator whose only reduction is a maximum (quantizers, division, transpose, dequantize, SiLU / Mul / Add
    forward and backward, GELU forward): FP8 codes, stored scales and bf16 results BIT-IDENTICAL, mismatch count 0;
    GELU backward: <= 1e-4 of the codes one step apart (another erff, see the test);
  * RMSNorm forward and LayerNorm forward without parameters: the CUDA kernels add the row sums in the order the
    reference's compiled kernels do (and contract the same multiply-adds), so mean, rstd, per-tensor scale and
    every code are BIT-IDENTICAL too, for rows of 16 ... 16384 elements, powers of two or not;
  * LayerNorm forward with weight and bias (the reference's kernel sums in another layout there) and the LayerNorm
    backward: rstd within 4 fp32 ulps, per-tensor scale equal or one bf16 step apart, and, when the scales are
    equal, >= 99.9 % identical codes, never more than one code step apart; dx within one bf16 step;
  * FP8 GEMM (accumulation order differs): |ours - reference| <= 2^-7 |ref| + 2^-7 rms(ref).
Shapes are reference-legal (both dimensions multiples of 256; its kernels have no boundary masks): a small one,
the activation benchmark tensor (8192 x 4096, seed 1, 0.1 % of the entries x100) and the Llama-2-7B MLP
activation (8192 x 11008).  The reference's RMSNorm / parametrised-LayerNorm BACKWARD kernels are not run: they
serialise through a device-side spin lock without a bound (func_rmsnorm.py:186-196, func_layernorm_param.py:199-211).
Each autotuned reference kernel runs with ONE of its own candidate configurations (tests/_ref.py).
"""
import pytest
import torch

from _ref import load_ref_triton, ref_module

pytestmark = pytest.mark.gpu
QB = 16
E4M3, E5M2 = torch.float8_e4m3fn, torch.float8_e5m2

SHAPES = {"small": (256, 512), "act": (8192, 4096), "mlp": (8192, 11008)}


def REF():
    ref = load_ref_triton()
    if ref is None:
        pytest.skip("oracle/_ref/coat_ref not staged (python oracle/build_ref.py)")
    return ref


def OURS():
    import coat_b200.activation.real_quantization as r
    return r


_CACHE = {}


def tensor(kind, seed, scale=1.0, outliers=True):
    """Seeded bf16 tensor, generated on the CPU and copied (cached per test session)."""
    key = (kind, seed, scale, outliers)
    if key not in _CACHE:
        M, N = SHAPES[kind]
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(M, N, generator=gen)
        if outliers:
            x[torch.rand(M, N, generator=gen) < 1e-3] *= 100
        _CACHE[key] = (x * scale).to(torch.bfloat16).cuda()
    return _CACHE[key]


def _bits(t):
    t = t.contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def mismatches(a, b):
    assert a.shape == b.shape and a.dtype == b.dtype, (a.shape, b.shape, a.dtype, b.dtype)
    return int((_bits(a) != _bits(b)).sum().item())


def same(name, a, b):
    n = mismatches(a, b)
    print(f"PARITY {name}: {n} mismatches of {a.numel()}")
    assert n == 0, f"{name}: {n} of {a.numel()} elements differ from the reference's kernel"


def code_steps(a, b):
    return (_bits(a).to(torch.int16) - _bits(b).to(torch.int16)).abs()


def ulps32(a, b):
    ia, ib = a.contiguous().view(torch.int32).long(), b.contiguous().view(torch.int32).long()
    return (ia - ib).abs().max().item()


def quantized(kind, seed, scale=1.0, fmt="E4M3"):
    """(codes, 1x16 scales) of a seeded tensor, produced by the REFERENCE's quantizer."""
    return REF().fp8_quantize(tensor(kind, seed, scale), QB, fmt)


# ------------------------------------------------------------------------------------------------------
# quantizers
# ------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("kind", ["small", "act", "mlp"])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("sdt", [torch.bfloat16, torch.float32])
def test_quantize(kind, fmt, sdt):
    x = tensor(kind, 1)
    y, s = OURS().fp8_quantize(x, QB, fmt, sdt)
    ry, rs = REF().fp8_quantize(x, QB, fmt, sdt)
    same(f"fp8_quantize[{kind},{fmt},{sdt}] codes", y, ry)
    same(f"fp8_quantize[{kind},{fmt},{sdt}] scales", s, rs)


@pytest.mark.parametrize("kind", ["small", "act", "mlp"])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("sdt", [torch.bfloat16, torch.float32])
def test_quantize_pertensor(kind, fmt, sdt):
    x = tensor(kind, 1)
    y, s_max, s = OURS().fp8_quantize_pertensor(x, QB, fmt, scale_dtype=sdt)
    ry, rs_max, rs = REF().fp8_quantize_pertensor(x, QB, fmt, scale_dtype=sdt)
    same("pertensor s_max", s_max, rs_max)
    same("pertensor group scales", s, rs)
    same(f"fp8_quantize_pertensor[{kind},{fmt},{sdt}] codes", y, ry)


@pytest.mark.parametrize("kind", ["small", "act", "mlp"])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_quantize_pertensor_transpose(kind, fmt):
    x = tensor(kind, 1)
    q, s_max, q_t = OURS().fp8_quantize_pertensor_transpose(x, QB, fmt)
    rq, rs_max, rq_t = REF().fp8_quantize_pertensor_transpose(x, QB, fmt)
    same("pertensor_transpose s_max", s_max, rs_max)
    same(f"fp8_quantize_pertensor_transpose[{kind},{fmt}] codes", q, rq)
    same(f"fp8_quantize_pertensor_transpose[{kind},{fmt}] transposed codes", q_t, rq_t)


@pytest.mark.parametrize("kind", ["small", "act"])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_division(kind, fmt):
    x = tensor(kind, 2)
    # default scale (computed by torch in the reference, _division.py:178-179) and a given bf16 / fp32 scale
    y, s = OURS().fp8_division(x, QB, fmt)
    ry, rs = REF().fp8_division(x, QB, fmt)
    same("division default scale", s, rs)
    same(f"fp8_division[{kind},{fmt}] codes", y, ry)
    for given in (rs * 1.37, rs.float() * 0.731):
        y, _ = OURS().fp8_division(x, QB, fmt, given)
        ry, _ = REF().fp8_division(x, QB, fmt, given)
        same(f"fp8_division[{kind},{fmt},{given.dtype}] codes", y, ry)
        q, _, q_t = OURS().fp8_division_transpose(x, QB, fmt, given)
        rq, _, rq_t = REF().fp8_division_transpose(x, QB, fmt, given)
        same(f"fp8_division_transpose[{kind},{fmt}] codes", q, rq)
        same(f"fp8_division_transpose[{kind},{fmt}] transposed", q_t, rq_t)
        q_t, _ = OURS().fp8_division_transpose(x, QB, fmt, given, only_transposed=True)
        same(f"fp8_division_transpose[{kind},{fmt}] only_transposed", q_t, rq_t)


@pytest.mark.parametrize("kind", ["small", "act", "mlp"])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("sdt", [torch.bfloat16, torch.float32])
def test_quantize_transpose(kind, fmt, sdt):
    x = tensor(kind, 1)
    (y, s), (y_t, s_t) = OURS().fp8_quantize_transpose(x, QB, fmt, sdt)
    (ry, rs), (ry_t, rs_t) = ref_module("_quantize_transpose").fp8_quantize_transpose(x, QB, fmt, sdt)
    same(f"fp8_quantize_transpose[{kind},{fmt},{sdt}] codes", y, ry)
    same("quantize_transpose scales", s, rs)
    same("quantize_transpose transposed codes", y_t, ry_t)
    same("quantize_transpose transposed scales", s_t, rs_t)


@pytest.mark.parametrize("kind", ["small", "act"])
def test_transpose_and_dequantize(kind):
    q, s = quantized(kind, 3)
    same("fp8_transpose", OURS().fp8_transpose(q), REF().fp8_transpose(q))
    same("fp8_dequantize", OURS().fp8_dequantize(q, s, QB), REF().fp8_dequantize(q, s, QB))


# ------------------------------------------------------------------------------------------------------
# fused quantize-on-save operators without a sum
# ------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("kind", ["small", "mlp"])
def test_silu_forward(kind):
    q, s = quantized(kind, 4, scale=2.0)
    y, s_y = OURS().fp8_silu_forward(q, s, QB)
    ry, rs_y = REF().fp8_silu_forward(q, s, QB)
    same(f"fp8_silu_forward[{kind}] scales", s_y, rs_y)
    same(f"fp8_silu_forward[{kind}] codes", y, ry)


@pytest.mark.parametrize("kind", ["small", "mlp"])
def test_silu_backward(kind):
    q, s = quantized(kind, 4, scale=2.0)
    g = tensor(kind, 5, scale=1e-2, outliers=False)
    y, s_y = OURS().fp8_silu_backward(q, s, g, QB, "E5M2")
    ry, rs_y = REF().fp8_silu_backward(q, s, g, QB, "E5M2")
    same(f"fp8_silu_backward[{kind}] bf16", y, ry)
    same(f"fp8_silu_backward[{kind}] scales", s_y, rs_y)
    qy, s_max, qy_t = OURS().fp8_silu_backward(q, s, g, QB, "E5M2", output_quantized_transpose=True)
    rqy, rs_max, rqy_t = REF().fp8_silu_backward(q, s, g, QB, "E5M2", output_quantized_transpose=True)
    same("silu_backward s_max", s_max, rs_max)
    same(f"fp8_silu_backward[{kind}] per-tensor codes", qy, rqy)
    same(f"fp8_silu_backward[{kind}] transposed codes", qy_t, rqy_t)


@pytest.mark.parametrize("kind", ["small", "mlp"])
def test_gelu_forward(kind):
    q, s = quantized(kind, 6, scale=2.0)
    qy, s_max, qy_t = OURS().fp8_gelu_forward(q, s, QB)
    rqy, rs_max, rqy_t = REF().fp8_gelu_forward(q, s, QB)
    same("gelu_forward s_max", s_max, rs_max)
    same(f"fp8_gelu_forward[{kind}] codes", qy, rqy)
    same(f"fp8_gelu_forward[{kind}] transposed codes", qy_t, rqy_t)


@pytest.mark.parametrize("kind", ["small", "mlp"])
def test_gelu_backward(kind):
    q, s = quantized(kind, 6, scale=2.0)
    g = tensor(kind, 7, scale=1e-2, outliers=False)
    qy, s_max = OURS().fp8_gelu_backward(q, s, g, QB, "E5M2")
    rqy, rs_max = REF().fp8_gelu_backward(q, s, g, QB, "E5M2")
    same("gelu_backward s_max", s_max, rs_max)
    # The one operator that is not bit-identical: for x < -3.9 the derivative is the small difference of
    # (1 + erf(x / sqrt 2)) / 2 and |x| pdf(x), and the erff that Triton links (its bundled libdevice) and the erff
    # of the CUDA 12.9 toolkit are different polynomials that disagree in the last place there.  Observed: 4e-5 of
    # the codes, all for x in [-5.6, -3.9].  Bound: 1e-4 of the codes, one code step.
    n = mismatches(qy, rqy)
    print(f"PARITY fp8_gelu_backward[{kind}] codes: {n} mismatches of {qy.numel()}")
    assert n <= 1e-4 * qy.numel() and code_steps(qy, rqy).max().item() <= 1


@pytest.mark.parametrize("kind", ["small", "mlp"])
def test_mul_forward(kind):
    q1, s1 = quantized(kind, 8)
    q2, s2 = quantized(kind, 9, scale=3.0)
    qy, s_max, qy_t = OURS().fp8_mul_forward(q1, s1, q2, s2, QB)
    rqy, rs_max, rqy_t = REF().fp8_mul_forward(q1, s1, q2, s2, QB)
    same("mul_forward s_max", s_max, rs_max)
    same(f"fp8_mul_forward[{kind}] codes", qy, rqy)
    same(f"fp8_mul_forward[{kind}] transposed codes", qy_t, rqy_t)


@pytest.mark.parametrize("kind", ["small", "mlp"])
def test_mul_backward(kind):
    q1, s1 = quantized(kind, 8)
    q2, s2 = quantized(kind, 9, scale=3.0)
    g = tensor(kind, 10, scale=1e-2, outliers=False)
    y1, (y2, s_y2) = OURS().fp8_mul_backward(q1, s1, q2, s2, g, QB, "E5M2")
    ry1, (ry2, rs_y2) = REF().fp8_mul_backward(q1, s1, q2, s2, g, QB, "E5M2")
    same(f"fp8_mul_backward[{kind}] y1", y1, ry1)
    same(f"fp8_mul_backward[{kind}] y2", y2, ry2)
    same(f"fp8_mul_backward[{kind}] scales", s_y2, rs_y2)
    y1, (qy2, s_max, qy2_t) = OURS().fp8_mul_backward(q1, s1, q2, s2, g, QB, "E5M2", output_quantized_transpose=True)
    ry1, (rqy2, rs_max, rqy2_t) = REF().fp8_mul_backward(q1, s1, q2, s2, g, QB, "E5M2",
                                                        output_quantized_transpose=True)
    same("mul_backward s_max", s_max, rs_max)
    same(f"fp8_mul_backward[{kind}] per-tensor codes", qy2, rqy2)
    same(f"fp8_mul_backward[{kind}] transposed codes", qy2_t, rqy2_t)


@pytest.mark.parametrize("kind", ["small", "act"])
def test_add(kind):
    a, b = tensor(kind, 11), tensor(kind, 12, scale=0.5)
    y1, (y2, s2) = OURS().fp8_add_Ifp_Ifp_Ofp_Og16(a, b, E4M3, QB)
    ry1, (ry2, rs2) = REF().fp8_add_Ifp_Ifp_Ofp_Og16(a, b, E4M3, QB)
    same(f"fp8_add_Og16[{kind}] sum", y1, ry1)
    same(f"fp8_add_Og16[{kind}] codes", y2, ry2)
    same(f"fp8_add_Og16[{kind}] scales", s2, rs2)
    y1, (q, s_max, s) = OURS().fp8_add_Ifp_Ifp_Ofp_Opt(a, b, QB, "E5M2")
    ry1, (rq, rs_max, rs) = REF().fp8_add_Ifp_Ifp_Ofp_Opt(a, b, QB, "E5M2")
    same(f"fp8_add_Opt[{kind}] sum", y1, ry1)
    same("add_Opt s_max", s_max, rs_max)
    same(f"fp8_add_Opt[{kind}] codes", q, rq)
    same(f"fp8_add_Opt[{kind}] group scales", s, rs)


@pytest.mark.parametrize("kind", ["small", "mlp"])
def test_gated_product_one_kernel_forms_equal_the_reference_pairs(kind):
    """The two extensions that run the gated product's operator pairs as one kernel, against the pairs of
    REFERENCE operators they stand for."""
    gate_q, gate_s = quantized(kind, 13, scale=2.0)
    up_q, up_s = quantized(kind, 14)
    g = tensor(kind, 15, scale=1e-2, outliers=False)
    (silu_q, silu_s), (mul_q, s_max, mul_q_t) = OURS().fp8_silu_mul_forward(gate_q, gate_s, up_q, up_s, QB)
    r_silu_q, r_silu_s = REF().fp8_silu_forward(gate_q, gate_s, QB)
    r_mul_q, r_s_max, r_mul_q_t = REF().fp8_mul_forward(r_silu_q, r_silu_s, up_q, up_s, QB)
    same("silu_mul_forward silu codes", silu_q, r_silu_q)
    same("silu_mul_forward silu scales", silu_s, r_silu_s)
    same("silu_mul_forward s_max", s_max, r_s_max)
    same(f"fp8_silu_mul_forward[{kind}] codes", mul_q, r_mul_q)
    same(f"fp8_silu_mul_forward[{kind}] transposed codes", mul_q_t, r_mul_q_t)

    (d_up, s_up, d_up_t), (d_gate, s_gate, d_gate_t) = OURS().fp8_mul_silu_backward(
        r_silu_q, r_silu_s, up_q, up_s, gate_q, gate_s, g, QB, "E5M2")
    r_y1, (r_d_up, r_s_up, r_d_up_t) = REF().fp8_mul_backward(r_silu_q, r_silu_s, up_q, up_s, g, QB, "E5M2",
                                                             output_quantized_transpose=True)
    r_d_gate, r_s_gate, r_d_gate_t = REF().fp8_silu_backward(gate_q, gate_s, r_y1, QB, "E5M2",
                                                            output_quantized_transpose=True)
    same("mul_silu_backward up scale", s_up, r_s_up)
    same(f"fp8_mul_silu_backward[{kind}] up codes", d_up, r_d_up)
    same(f"fp8_mul_silu_backward[{kind}] up transposed", d_up_t, r_d_up_t)
    same("mul_silu_backward gate scale", s_gate, r_s_gate)
    same(f"fp8_mul_silu_backward[{kind}] gate codes", d_gate, r_d_gate)
    same(f"fp8_mul_silu_backward[{kind}] gate transposed", d_gate_t, r_d_gate_t)


# ------------------------------------------------------------------------------------------------------
# norms (sum order differs: tolerances of the module docstring)
# ------------------------------------------------------------------------------------------------------
def _norm_outputs_close(name, mine, ref, rstd_ulps):
    (qy, s_max, qy_t, rstd), (rqy, rs_max, rqy_t, r_rstd) = mine, ref
    u = ulps32(rstd, r_rstd)
    print(f"PARITY {name}: rstd max {u} ulps")
    assert u <= rstd_ulps
    a, b = s_max.float().item(), rs_max.float().item()
    assert abs(a - b) <= b * 2 ** -7 * 1.01, (a, b)
    assert torch.equal(_bits(qy).t(), _bits(qy_t))
    if a == b:
        n = mismatches(qy, rqy)
        print(f"PARITY {name}: {n} mismatches of {qy.numel()} codes, scales equal")
        assert n <= 1e-3 * qy.numel() and code_steps(qy, rqy).max().item() <= 1
    else:
        print(f"PARITY {name}: per-tensor scales one bf16 step apart ({a} vs {b}); codes not compared")


def _norm_input(M, N, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, N, generator=gen)
    x[torch.rand(M, N, generator=gen) < 1e-3] *= 100
    x += 0.25   # a non-zero mean, so that the LayerNorm's first sum matters
    return REF().fp8_quantize(x.to(torch.bfloat16).cuda(), QB, "E4M3")


NORM_SHAPES = [(256, 256), (256, 512), (256, 1024), (256, 2048), (8192, 4096), (256, 8192), (256, 11008), (256, 16384),
               (256, 768), (256, 5120)]


@pytest.mark.parametrize("M,N", NORM_SHAPES)
def test_rmsnorm_forward(M, N):
    q, s = _norm_input(M, N, 16)
    w = (1 + 0.1 * torch.randn(N, generator=torch.Generator().manual_seed(17))).to(torch.bfloat16).cuda()
    qy, s_max, qy_t, (_, rstd, _) = OURS().fp8_rmsnorm_forward(q, s, w, QB, 1e-5)
    rqy, rs_max, rqy_t, (_, r_rstd, _) = REF().fp8_rmsnorm_forward(q, s, w, QB, 1e-5)
    same(f"fp8_rmsnorm_forward[{M}x{N}] rstd", rstd, r_rstd)
    same(f"fp8_rmsnorm_forward[{M}x{N}] s_max", s_max, rs_max)
    same(f"fp8_rmsnorm_forward[{M}x{N}] codes", qy, rqy)
    same(f"fp8_rmsnorm_forward[{M}x{N}] transposed codes", qy_t, rqy_t)


@pytest.mark.parametrize("M,N", NORM_SHAPES)
def test_layernorm_noparam_forward(M, N):
    q, s = _norm_input(M, N, 18)
    qy, s_max, qy_t, (mean, rstd, _) = OURS().fp8_layernorm_noparam_forward(q, s, QB, 1e-5)
    rqy, rs_max, rqy_t, (r_mean, r_rstd, _) = REF().fp8_layernorm_noparam_forward(q, s, QB, 1e-5)
    same(f"fp8_layernorm_noparam_forward[{M}x{N}] mean", mean, r_mean)
    same(f"fp8_layernorm_noparam_forward[{M}x{N}] rstd", rstd, r_rstd)
    same(f"fp8_layernorm_noparam_forward[{M}x{N}] s_max", s_max, rs_max)
    same(f"fp8_layernorm_noparam_forward[{M}x{N}] codes", qy, rqy)
    same(f"fp8_layernorm_noparam_forward[{M}x{N}] transposed codes", qy_t, rqy_t)


@pytest.mark.parametrize("M,N", [(256, 512), (8192, 4096)])
def test_layernorm_param_forward(M, N):
    q, s = _norm_input(M, N, 18)
    gen = torch.Generator().manual_seed(19)
    w = (1 + 0.1 * torch.randn(N, generator=gen)).to(torch.bfloat16).cuda()
    b = (0.1 * torch.randn(N, generator=gen)).to(torch.bfloat16).cuda()
    qy, s_max, qy_t, (_, _, mean, rstd, _) = OURS().fp8_layernorm_param_forward(q, s, w, b, QB, 1e-5)
    rqy, rs_max, rqy_t, (_, _, r_mean, r_rstd, _) = REF().fp8_layernorm_param_forward(q, s, w, b, QB, 1e-5)
    assert (mean - r_mean).abs().max().item() <= 1e-6
    _norm_outputs_close(f"fp8_layernorm_param_forward[{M}x{N}]", (qy, s_max, qy_t, rstd),
                        (rqy, rs_max, rqy_t, r_rstd), 4)


@pytest.mark.parametrize("M,N", [(256, 512), (8192, 4096)])
def test_layernorm_noparam_backward(M, N):
    """The one norm backward of the reference without a spin lock.  bf16 dx: the two row sums are added in another
    order, so dx may differ by one bf16 step of its own size plus a rounding of the row-wide terms that cancel in it
    (2^-9 of the row's largest |dx|); identical in >= 99 % of the places."""
    q, s = _norm_input(M, N, 18)
    g = (torch.randn(M, N, generator=torch.Generator().manual_seed(20)) * 1e-2).to(torch.bfloat16).cuda()
    _, _, _, (mean, rstd, nw) = REF().fp8_layernorm_noparam_forward(q, s, QB, 1e-5)
    dx = OURS().fp8_layernorm_noparam_backward(q, s, g, QB, mean, rstd, nw)
    rdx = REF().fp8_layernorm_noparam_backward(q, s, g, QB, mean, rstd, nw)
    n = mismatches(dx, rdx)
    print(f"PARITY fp8_layernorm_noparam_backward[{M}x{N}]: {n} mismatches of {dx.numel()}")
    assert n <= 1e-2 * dx.numel()
    err = (dx.float() - rdx.float()).abs()
    bound = rdx.float().abs() * 2 ** -7 + rdx.float().abs().amax(dim=1, keepdim=True) * 2 ** -9
    assert bool((err <= bound).all())


# ------------------------------------------------------------------------------------------------------
# FP8 GEMM / linear
# ------------------------------------------------------------------------------------------------------
def _gemm_close(name, y, ry):
    y, ry = y.float(), ry.float()
    rms = ry.pow(2).mean().sqrt()
    err = (y - ry).abs()
    bad = int((err > 2 ** -7 * ry.abs() + 2 ** -7 * rms).sum().item())
    print(f"PARITY {name}: {bad} of {y.numel()} outside tolerance, max err {err.max().item():.3e}, rms {rms.item():.3e}, "
          f"{int((y != ry).sum().item())} not identical")
    assert bad == 0


@pytest.mark.parametrize("shape", ["small", "llama_mlp"])
@pytest.mark.parametrize("gfmt", ["E5M2", "E4M3"])
def test_linear_forward_backward(shape, gfmt):
    """FP8Linear's three GEMMs as the reference composes them (fp8linear.py:64-110): per-tensor codes and their
    transposes from fp8_quantize_pertensor_transpose, gradients in E5M2 (the default) or E4M3."""
    M, K, N = (256, 512, 768) if shape == "small" else (8192, 4096, 11008)
    gen = torch.Generator().manual_seed(2)
    X = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    W = (torch.randn(N, K, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    G = (torch.randn(M, N, generator=gen) * 1e-2).to(torch.bfloat16).cuda()
    ref = REF()
    qx, sx, qx_t = ref.fp8_quantize_pertensor_transpose(X, QB, "E4M3")
    qw, sw, qw_t = ref.fp8_quantize_pertensor_transpose(W, QB, "E4M3")
    qg, sg, qg_t = ref.fp8_quantize_pertensor_transpose(G, QB, gfmt)
    _gemm_close(f"fp8_linear_forward[{shape}]", OURS().fp8_linear_forward(qx, sx, qw, sw, False, QB),
                ref.fp8_linear_forward(qx, sx, qw, sw, False, QB))
    bias = (torch.randn(N, generator=gen) * 0.1).to(torch.bfloat16).cuda()
    _gemm_close(f"fp8_linear_forward+bias[{shape}]", OURS().fp8_linear_forward(qx, sx, qw, sw, False, QB, bias),
                ref.fp8_linear_forward(qx, sx, qw, sw, False, QB, bias))
    dx, dw = OURS().fp8_linear_backward(qx_t, sx, qg, sg, qg_t, qw_t, sw, QB)
    rdx, rdw = ref.fp8_linear_backward(qx_t, sx, qg, sg, qg_t, qw_t, sw, QB)
    _gemm_close(f"fp8_linear_backward[{shape},{gfmt}] dgrad", dx, rdx)
    _gemm_close(f"fp8_linear_backward[{shape},{gfmt}] wgrad", dw, rdw)
    # quantising epilogue: codes x scales compared as values (one E4M3 step where the accumulations differ)
    (y, s_y), (ry, rs_y) = (OURS().fp8_linear_forward(qx, sx, qw, sw, True, QB),
                            ref.fp8_linear_forward(qx, sx, qw, sw, True, QB))
    assert y.dtype == ry.dtype and s_y.dtype == rs_y.dtype and s_y.shape == rs_y.shape
    n_s, n_c = mismatches(s_y, rs_y), mismatches(y, ry)
    print(f"PARITY fp8_linear_forward[{shape}] quantising epilogue: {n_s} of {s_y.numel()} scales, "
          f"{n_c} of {y.numel()} codes differ")
    assert n_s <= 0.02 * s_y.numel() and n_c <= 0.05 * y.numel()
    dq = lambda c, s: c.float().view(M, -1, QB) * s.float().unsqueeze(-1)
    err = (dq(y, s_y) - dq(ry, rs_y)).abs()
    assert bool((err <= dq(ry, rs_y).abs() * 2 ** -3 + rs_y.float().unsqueeze(-1) * 2 ** -6).all())


# ------------------------------------------------------------------------------------------------------
# 128-granular (block-scaled recipe) quantizers
# ------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("kind", ["small", "act"])
@pytest.mark.parametrize("sdt", [torch.float32, torch.bfloat16])
def test_block128_quantizers(kind, sdt):
    x = tensor(kind, 21)
    y, s = OURS().fp8_quantize_perblock(x, 128, "E4M3", sdt)
    ry, rs = REF().fp8_quantize_perblock(x, 128, "E4M3", sdt)
    same(f"fp8_quantize_perblock[{kind},{sdt}] codes", y, ry)
    same("perblock scales", s, rs.reshape(s.shape))
    (y, s), (y_t, s_t) = OURS().fp8_quantize_perblock_transpose(x, 128, "E4M3", sdt)
    (ry, rs), (ry_t, rs_t) = ref_module("_quantize_perblock_transpose").fp8_quantize_perblock_transpose(
        x, 128, "E4M3", sdt)
    same("perblock_transpose codes", y, ry)
    same("perblock_transpose scales", s, rs.reshape(s.shape))
    same("perblock_transpose transposed codes", y_t, ry_t)
    same("perblock_transpose transposed scales", s_t, rs_t.reshape(s_t.shape))
    (y, s), (y_t, s_t), (y_g, s_g) = OURS().fp8_quantize_perblock_transpose_pergroup(x, 128, "E4M3", sdt)
    (ry, rs), (ry_t, rs_t), (ry_g, rs_g) = ref_module(
        "_quantize_perblock_transpose_pergroup").fp8_quantize_perblock_transpose_pergroup(x, 128, "E4M3", sdt)
    same("perblock_transpose_pergroup codes", y, ry)
    same("perblock_transpose_pergroup transposed codes", y_t, ry_t)
    same("perblock_transpose_pergroup row-group codes", y_g, ry_g)
    same("perblock_transpose_pergroup row-group scales", s_g, rs_g.reshape(s_g.shape))
    (y, s), (y_t, s_t) = OURS().fp8_quantize_transpose(x, 128, "E4M3", sdt)
    (ry, rs), (ry_t, rs_t) = ref_module("_quantize_transpose").fp8_quantize_transpose(x, 128, "E4M3", sdt)
    same("quantize_transpose QB=128 codes", y, ry)
    same("quantize_transpose QB=128 scales", s, rs)
    same("quantize_transpose QB=128 transposed codes", y_t, ry_t)
    same("quantize_transpose QB=128 transposed scales", s_t, rs_t)
