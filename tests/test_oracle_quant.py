"""CPU tests of the quantizer restatement (oracle/quant.py) against golden vectors made from the
reference's own pure-PyTorch expectation, plus structural properties."""
import os

import numpy as np
import pytest
import torch

from oracle import quant as Q

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz")
BS, SL, CDIM, QB = 2, 32, 128, 16


def similarity(a, b):
    return (a == b).float().mean().item()


@pytest.mark.parametrize("seed", [0, 1])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_per_group_against_reference_expectation(seed, fmt):
    """The reference's criterion (tests/test_utils.py:98-119, used e.g. by tests/test_fp8_quantize.py):
    at least 95 % of the dequantised elements exactly equal.  The expectation divides by the bf16-rounded
    scale and adds no 1e-10; the kernels (and this restatement) divide by the fp32 scale."""
    z = np.load(GOLDEN)
    x = torch.from_numpy(z[f"s{seed}/x"]).reshape(-1, CDIM)
    q, s = Q.fp8_quantize(x, QB, fmt)
    rq = Q.fp8_dequantize(q, s, QB).float()
    # dequantised with the same bf16 scales as the expectation
    exp_rq = torch.from_numpy(z[f"s{seed}/{fmt}/per_group/rqx"]).reshape(-1, CDIM)
    exp_s = torch.from_numpy(z[f"s{seed}/{fmt}/per_group/sx"]).reshape(-1, CDIM // QB)
    assert similarity(s.float(), exp_s) >= 0.95
    mine = (q.float().reshape(-1, CDIM // QB, QB) * s.float().unsqueeze(-1)).reshape(-1, CDIM)
    assert similarity(mine, exp_rq) >= 0.95
    assert (rq - x).abs().max() <= x.abs().max() / (8 if fmt == "E4M3" else 4)


@pytest.mark.parametrize("seed", [0, 1])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
def test_per_tensor_against_reference_expectation(seed, fmt):
    z = np.load(GOLDEN)
    x = torch.from_numpy(z[f"s{seed}/x"]).reshape(-1, CDIM)
    q, s_max, s_y = Q.fp8_quantize_pertensor(x, QB, fmt)
    exp_s = torch.from_numpy(z[f"s{seed}/{fmt}/per_tensor/sx"])
    exp_q = torch.from_numpy(z[f"s{seed}/{fmt}/per_tensor/qx"]).reshape(-1, CDIM)
    # one bf16 scale for the tensor: equal, or one bf16 step apart (the 1e-10 and rounding order)
    assert abs(s_max.float().item() - exp_s.item()) <= exp_s.item() * 2 ** -7
    if s_max.float().item() == exp_s.item():
        assert similarity(q.view(torch.uint8), exp_q) >= 0.95
    assert s_y.max() == s_max and s_y.shape == (BS * SL, CDIM // QB)


def test_transposed_outputs_are_consistent():
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(64, 96, generator=gen).to(torch.bfloat16)
    (y, s_y), (y_t, s_y_t) = Q.fp8_quantize_transpose(x, 16, "E4M3")
    assert y.shape == (64, 96) and y_t.shape == (96, 64) and s_y.shape == (64, 6) and s_y_t.shape == (96, 4)
    # the transposed half is the straight quantizer applied to x^T
    y2, s2 = Q.fp8_quantize(x.t().contiguous(), 16, "E4M3")
    assert torch.equal(y_t.view(torch.uint8), y2.view(torch.uint8)) and torch.equal(s_y_t, s2)
    q, s_max, q_t = Q.fp8_quantize_pertensor_transpose(x, 16, "E4M3")
    assert torch.equal(q.view(torch.uint8).t(), q_t.view(torch.uint8))


def test_saturation_and_zero_groups():
    x = torch.zeros(4, 32)
    x[1, :16] = torch.linspace(-3, 3, 16)
    x[2, 5] = 1e30
    q, s = Q.fp8_quantize(x, 16, "E4M3", scale_dtype=torch.float32)
    assert torch.equal(s[0], torch.full((2,), 1e-10 / 448))          # all-zero group: scale is 1e-10/448
    assert (q[0].view(torch.uint8) == 0).all()
    assert q[1, 15].float() == 448 and q[1, 0].float() == -448      # the group maximum maps to +-448
    assert q[2, 5].float() == 448 and not q.float().isnan().any()
