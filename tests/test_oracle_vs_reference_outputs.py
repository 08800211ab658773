"""Pins the torch restatements under oracle/ (quant.py, fused.py, gemm.py) to OUTPUTS OF THE REFERENCE ITSELF: its
Triton kernels, run on a B200 by tests/golden/make_triton_golden.py on small seeded inputs and stored in
tests/golden/triton_golden.npz.  Runs on the CPU.

The restatements divide with IEEE division, the reference's compiled kernels with the GPU's approximate full-range
division (<= 2 ulp), and libm stands in for libdevice: so a code may differ where the quotient lies within a few
fp32 ulps of a rounding boundary (with bf16 inputs mostly exact ties).  Criterion, fixed up front: maximum-only
operators >= 99.8 % of the codes identical and never more than one code step apart, bf16 scales identical except
<= 1 % one bf16 step apart (exact ties of the un-rounded scale), fp32 scales within 2 ulps; bf16 results identical in >= 99.5 % and within one bf16
step; sums (norms, GEMM) as stated per test."""
import os

import numpy as np
import pytest
import torch

from oracle import fused as F
from oracle import gemm as G
from oracle import quant as Q

QB = 16
E4M3, E5M2 = torch.float8_e4m3fn, torch.float8_e5m2
PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "triton_golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(PATH)


def f8(arr, fmt):
    return torch.from_numpy(arr.copy()).view(E4M3 if fmt == "E4M3" else E5M2)


def bf(arr):
    return torch.from_numpy(arr.copy()).to(torch.bfloat16)


def codes_close(mine, ref_bytes, min_equal=0.998):
    a = mine.contiguous().view(torch.uint8).to(torch.int16)
    b = torch.from_numpy(ref_bytes.copy()).to(torch.int16)
    assert a.shape == b.shape
    assert (a == b).float().mean().item() >= min_equal, (a != b).sum().item()
    assert (a - b).abs().max().item() <= 1


def bf16_close(mine, ref_vals, min_equal=0.995):
    a, b = mine.float(), torch.from_numpy(ref_vals.copy())
    assert a.shape == b.shape
    assert (a == b).float().mean().item() >= min_equal
    assert bool(((a - b).abs() <= b.abs() * 2 ** -7 + 1e-38).all())


def scales_close(mine, ref_vals, fp32=False):
    a, b = mine.float(), torch.from_numpy(ref_vals.copy())
    assert a.shape == b.shape
    if fp32:
        assert bool(((a - b).abs() <= b.abs() * 2 ** -22).all())
    else:
        assert (a == b).float().mean().item() >= 0.99 and bool(((a - b).abs() <= b.abs() * 2 ** -7).all())


@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_quantizers(gold, fmt):
    x = bf(gold["x"])
    y, s = Q.fp8_quantize(x, QB, fmt)
    codes_close(y, gold[f"quantize/{fmt}/y"]), scales_close(s, gold[f"quantize/{fmt}/s"])
    y, s = Q.fp8_quantize(x, QB, fmt, torch.float32)
    codes_close(y, gold[f"quantize_f32/{fmt}/y"]), scales_close(s, gold[f"quantize_f32/{fmt}/s"], fp32=True)
    y, s_max, s = Q.fp8_quantize_pertensor(x, QB, fmt)
    assert s_max.float().item() == float(gold[f"pertensor/{fmt}/s_max"])
    codes_close(y, gold[f"pertensor/{fmt}/y"]), scales_close(s, gold[f"pertensor/{fmt}/s"])
    y, s_max, y_t = Q.fp8_quantize_pertensor_transpose(x, QB, fmt)
    assert s_max.float().item() == float(gold[f"pertensor_t/{fmt}/s_max"])
    codes_close(y, gold[f"pertensor_t/{fmt}/y"]), codes_close(y_t, gold[f"pertensor_t/{fmt}/y_t"])
    (y, s), (y_t, s_t) = Q.fp8_quantize_transpose(x, QB, fmt)
    codes_close(y, gold[f"quantize_t/{fmt}/y"]), scales_close(s, gold[f"quantize_t/{fmt}/s"])
    codes_close(y_t, gold[f"quantize_t/{fmt}/y_t"]), scales_close(s_t, gold[f"quantize_t/{fmt}/s_t"])
    given = torch.tensor(float(gold[f"division/{fmt}/s"]), dtype=torch.bfloat16)
    codes_close(Q.fp8_division(x, fmt, given), gold[f"division/{fmt}/y"])


def _inputs(gold):
    return (f8(gold["in/q"], "E4M3"), bf(gold["in/s"]), f8(gold["in/q2"], "E4M3"), bf(gold["in/s2"]), bf(gold["g"]))


def test_dequantize_and_activations(gold):
    q, s, q2, s2, g = _inputs(gold)
    bf16_close(Q.fp8_dequantize(q, s, QB), gold["dequantize/y"], min_equal=1.0)
    y, s_y = F.silu_forward(q, s, QB)
    codes_close(y, gold["silu_fwd/y"]), scales_close(s_y, gold["silu_fwd/s"])
    ey, es_y, es_max, eq, _ = F.per_tensor_from_value(F.silu_backward_value(q, s, g, QB), QB, "E5M2")
    bf16_close(ey, gold["silu_bwd/y"]), scales_close(es_y, gold["silu_bwd/s"])
    assert es_max.float().item() == float(gold["silu_bwd/s_max"])
    codes_close(eq, gold["silu_bwd/q"], min_equal=0.995)
    _, _, es_max, eq, _ = F.per_tensor_from_value(F.gelu_forward_value(q, s, QB), QB, "E4M3")
    assert es_max.float().item() == float(gold["gelu_fwd/s_max"])
    codes_close(eq, gold["gelu_fwd/q"], min_equal=0.995)
    _, _, es_max, eq, _ = F.per_tensor_from_value(F.gelu_backward_value(q, s, g, QB), QB, "E5M2")
    assert es_max.float().item() == float(gold["gelu_bwd/s_max"])
    codes_close(eq, gold["gelu_bwd/q"], min_equal=0.995)


def test_mul_and_add(gold):
    q, s, q2, s2, g = _inputs(gold)
    _, _, es_max, eq, eq_t = F.per_tensor_from_value(F.mul_forward_value(q, s, q2, s2, QB), QB, "E4M3")
    assert es_max.float().item() == float(gold["mul_fwd/s_max"])
    codes_close(eq, gold["mul_fwd/q"]), codes_close(eq_t, gold["mul_fwd/q_t"])
    v1, v2 = F.mul_backward_values(q, s, q2, s2, g, QB)
    bf16_close(v1.to(torch.bfloat16), gold["mul_bwd/y1"], min_equal=1.0)
    ey2, es_y2, _, _, _ = F.per_tensor_from_value(v2, QB, "E5M2")
    bf16_close(ey2, gold["mul_bwd/y2"], min_equal=1.0), scales_close(es_y2, gold["mul_bwd/s"])
    a, b = bf(gold["add/a"]), bf(gold["add/b"])
    y1, (y2, s_y2) = F.add_forward(a, b, "E4M3", QB)
    bf16_close(y1, gold["add_fwd/y1"], min_equal=1.0)
    codes_close(y2, gold["add_fwd/y2"]), scales_close(s_y2, gold["add_fwd/s"])
    bf16_close(y1, gold["add_bwd/y1"], min_equal=1.0)
    # add_bwd.py: group scales of the fp32 sum, their maximum, division of the bf16 sum by it
    s_g = Q.group_scales(a.float() + b.float(), QB, "E5M2").to(torch.bfloat16)
    scales_close(s_g, gold["add_bwd/s"])
    assert s_g.max().float().item() == float(gold["add_bwd/s_max"])
    codes_close(Q.fp8_division(y1, "E5M2", s_g.max()), gold["add_bwd/q"])


def test_norms(gold):
    """Row sums in another order than the reference's kernels: rstd / mean to 1e-6 relative (resp. of the row's
    scale), the per-tensor scale equal or one bf16 step apart, codes >= 99 % identical when it is equal."""
    q, s, _, _, g = _inputs(gold)
    w, b = bf(gold["norm/w"]), bf(gold["norm/b"])

    def check(value, stat, name):
        es_max = F.rmsnorm_row_scales(value, "E4M3").max()
        ref = float(gold[f"{name}/s_max"])
        assert abs(es_max.float().item() - ref) <= ref * 2 ** -7
        assert torch.allclose(stat, torch.from_numpy(gold[f"{name}/rstd"].copy()), rtol=2e-6, atol=0)
        if es_max.float().item() == ref:
            codes_close(Q.fp8_division(value, "E4M3", es_max), gold[f"{name}/q"], min_equal=0.99)

    value, rstd = F.rmsnorm_forward_value(q, s, w, QB, 1e-5)
    check(value.to(torch.bfloat16), rstd, "rmsnorm_fwd")
    value, mean, rstd = F.layernorm_forward_value(q, s, None, None, QB, 1e-5)
    amax = float(F.dequant(q, s, QB).abs().max())
    assert torch.allclose(mean, torch.from_numpy(gold["ln_noparam_fwd/mean"].copy()), rtol=0, atol=5e-7 * amax)
    check(value, rstd, "ln_noparam_fwd")
    dx, _, _ = F.layernorm_backward(q, s, g, None, torch.from_numpy(gold["ln_noparam_fwd/mean"].copy()),
                                    torch.from_numpy(gold["ln_noparam_fwd/rstd"].copy()), QB)
    ref = torch.from_numpy(gold["ln_noparam_bwd/dx"].copy())
    assert (dx.float() == ref).float().mean().item() >= 0.97
    assert bool(((dx.float() - ref).abs() <= ref.abs() * 2 ** -7 + ref.abs().amax(dim=1, keepdim=True) * 2 ** -9).all())
    value, mean, rstd = F.layernorm_forward_value(q, s, w, b, QB, 1e-5)
    check(value, rstd, "ln_param_fwd")


def test_gemm(gold):
    """The reference's Triton GEMM against exact arithmetic on the same codes and scales: within the GEMM tolerance
    (2^-7 |y| + 2^-7 rms(y)) that the CUDA GEMM is held to."""
    t = {k: gold[f"gemm/{k}"] for k in ("qx", "sx", "qx_t", "qw", "sw", "qw_t", "qg", "sg", "qg_t", "y", "dx", "dw")}
    sx, sw, sg = (torch.tensor(float(t[k]), dtype=torch.bfloat16) for k in ("sx", "sw", "sg"))
    y = G.fp8_matmul_fp64(f8(t["qx"], "E4M3"), f8(t["qw"], "E4M3"), sx, sw)
    assert bool(G.within_tolerance(torch.from_numpy(t["y"].copy()), y).all())
    dx = G.fp8_matmul_fp64(f8(t["qg"], "E5M2"), f8(t["qw_t"], "E4M3"), sg, sw)
    assert bool(G.within_tolerance(torch.from_numpy(t["dx"].copy()), dx).all())
    dw = G.fp8_matmul_fp64(f8(t["qg_t"], "E5M2"), f8(t["qx_t"], "E4M3"), sg, sx)
    assert bool(G.within_tolerance(torch.from_numpy(t["dw"].copy()), dw).all())
