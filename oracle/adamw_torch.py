"""Pure-PyTorch FP8 AdamW step with Dynamic Range Expansion on the CPU (TEST / BASELINE INFRASTRUCTURE ONLY).

A restatement, in this repository's own code, of the expectation the reference's optimizer test compares its kernel
with: `simulated_optimizer_expand_step` (tests/test_fp8_adamw_expand.py:111-215) with the torch fake-quantizer
(coat/activation/fake_quantization/quantize_function.py:226-262, `floatExMy_quantize_torch`, which equals
clamp + round-to-nearest-even cast to float8_e4m3fn) in place of the Triton one.  It is what "COAT's pure-PyTorch
reference path" means for the optimizer, and it is what bench.py times on the host cores as the second CPU baseline.

It is NOT the kernel's arithmetic; the known differences are kept as they are in the reference:
  * the expansion exponent is found by a table search over i/16, i = 1..128, with a strict `<` (so it is capped at 8
    and an index of zero wraps around to 8), not by the closed form floor(log2(UB) / log2(R) * 16) / 16;
  * the group minimum includes exact zeros; 1e-8 (not 1e-30) is added to the group maximum before the scale;
  * weight decay is decoupled (`p *= 1 - lr * wd` before the update), the kernel folds it into the update.
Pinned by tests/test_oracle_adamw.py against golden vectors made by executing the reference's test text
(tests/golden/make_adamw_golden.py).
"""
import math

import torch

GROUP = 128
RATIO_UPPER_BOUND = 448.0 * 448.0 / 2.0
EPSILON = 1e-8   # QArgs.epsilon, tests/test_fp8_adamw_expand.py:37


def _power_options(like):
    return torch.tensor([i / 16 for i in range(1, 129)], dtype=like.dtype)


def fake_quantize_e4m3(blocks):
    """block_quant(..., "E4M3") on [G, 128] blocks -> (dequantised, codes as floats, scale [G, 1])."""
    scale = (blocks.abs().amax(dim=1, keepdim=True) + EPSILON) / 448.0
    q = (blocks / scale).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn).to(blocks.dtype)
    return q * scale, q, scale


def dequantize_state(codes, scale, expand, sqrt_minmax):
    """What the reference's test feeds the step: sign(q s) |q s|^(1/k) r per group of 128 (:106-107)."""
    v = codes.view(torch.float8_e4m3fn).float().view(-1, GROUP) * scale.view(-1, 1)
    v = v.sign() * torch.pow(v.abs(), 1.0 / expand.view(-1, 1)) * sqrt_minmax.view(-1, 1)
    return v.view(-1)


def _expand_and_quantize(flat, signed):
    """Dynamic range expansion + fake quantisation of one moment (:133-176 / :178-213).
    -> (dequantised moment, codes, scale [G], exponent [G], sqrt(max * min) [G])."""
    blocks = flat.view(-1, GROUP)
    mag = blocks.abs() if signed else blocks
    sign = blocks.sign()
    bmax, bmin = mag.max(dim=1)[0], mag.min(dim=1)[0]
    sqrt_minmax = (bmax * bmin).sqrt().unsqueeze(1)
    ratio = (bmax / bmin).unsqueeze(1)
    options = _power_options(flat)
    idx = (torch.pow(ratio, options.unsqueeze(0)) < RATIO_UPPER_BOUND).sum(dim=1)
    exponent = options[idx - 1].unsqueeze(1)       # index 0 wraps to the last option, as in the reference
    centred = blocks / sqrt_minmax
    expanded = torch.pow(centred.abs(), exponent) * sign if signed else torch.pow(centred, exponent)
    rq, q, scale = fake_quantize_e4m3(expanded)
    back = torch.pow(rq.abs(), 1.0 / exponent)
    if signed:
        back = back * sign
    back = back * sqrt_minmax
    return back.reshape(-1), q.reshape(-1), scale.flatten(), exponent.flatten(), sqrt_minmax.flatten()


def pure_pytorch_expand_step(params, grads, exp_avg, exp_avg_sq, beta1, beta2, lr, wd, eps, step):
    """One step on flat fp32 tensors whose length is a multiple of 128; params, exp_avg and exp_avg_sq are updated in
    place (the moments to their dequantised values).  `step` is the count BEFORE this step, as in the reference's
    test.  Returns the quantised state: dict of codes (as floats), scales, exponents and sqrt(max*min) per moment."""
    step += 1
    params.mul_(1 - lr * wd)
    exp_avg.lerp_(grads, 1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(grads, grads, value=1 - beta2)
    bias_correction1 = 1 - beta1 ** step
    bias_correction2 = 1 - beta2 ** step
    step_size = lr / bias_correction1
    denom = (exp_avg_sq.sqrt() / math.sqrt(bias_correction2)).add_(eps)
    params.addcdiv_(exp_avg, denom, value=-step_size)
    m, q_m, s_m, k_m, r_m = _expand_and_quantize(exp_avg, signed=True)
    v, q_v, s_v, k_v, r_v = _expand_and_quantize(exp_avg_sq, signed=False)
    exp_avg.copy_(m)
    exp_avg_sq.copy_(v)
    return dict(q_m=q_m, s_m=s_m, k_m=k_m, r_m=r_m, q_v=q_v, s_v=s_v, k_v=k_v, r_v=r_v)
