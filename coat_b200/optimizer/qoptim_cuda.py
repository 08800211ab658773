"""Drop-in for the reference's native module `qoptim_cuda`
(coat/optimizer/kernels/bindings.cpp:5-8): same two functions, same positional
arguments, tensors updated in place, nothing returned.  The work is done by the
fused sm_100a kernels behind the C ABI (include/coat_b200.h)."""
import torch

from .. import _lib


def _check_state(name, t, groups):
    if t.dtype != torch.float32:
        # The reference reads these buffers as float* whatever their dtype
        # (fp8_adamw_expand_cuda_kernel.cu:234-240 via data_ptr<float>(), which throws).
        raise RuntimeError(f"expected scalar type Float but found {t.dtype} for {name}")
    if t.numel() != groups:
        raise RuntimeError(f"{name} must hold one value per 128-element group ({groups}), has {t.numel()}")


def fp8_adamw_expand_step(params, grads, exp_avg, scale_exp_avg, expand_exp_avg, sqrtminmax_exp_avg,
                          exp_avg_sq, scale_exp_avg_sq, expand_exp_avg_sq, sqrtminmax_exp_avg_sq,
                          beta1, beta2, lr, wd, eps, step, qgroup_size, expand_min, *, bf16_out=None, flags=0):
    """qoptim_cuda.fp8_adamw_expand_step (coat/optimizer/kernels/include/fp8_adamw_expand.h:6-17)."""
    if qgroup_size != 128:
        raise RuntimeError("Only Support 128 per-group quantization currently")
    n = params.numel()
    groups = (n + 127) // 128
    for nm, t in (("scale_exp_avg", scale_exp_avg), ("expand_exp_avg", expand_exp_avg),
                  ("sqrtminmax_exp_avg", sqrtminmax_exp_avg), ("scale_exp_avg_sq", scale_exp_avg_sq),
                  ("expand_exp_avg_sq", expand_exp_avg_sq), ("sqrtminmax_exp_avg_sq", sqrtminmax_exp_avg_sq)):
        _check_state(nm, t, groups)
    if grads.dtype != params.dtype or grads.numel() != n:
        raise RuntimeError("grads must match params in dtype and size")
    P = _lib.dev_ptr
    P(params, "params")  # raises for a CPU tensor before any device is selected
    with torch.cuda.device(params.device):
        rc = _lib.lib().coat_fp8_adamw_expand_step(
            P(params, "params"), P(grads, "grads"), P(exp_avg, "exp_avg"), P(scale_exp_avg),
            P(expand_exp_avg), P(sqrtminmax_exp_avg), P(exp_avg_sq, "exp_avg_sq"), P(scale_exp_avg_sq),
            P(expand_exp_avg_sq), P(sqrtminmax_exp_avg_sq), beta1, beta2, lr, wd, eps, int(step),
            int(qgroup_size), int(expand_min), n, _lib.param_dtype(params), P(bf16_out), int(flags),
            _lib.stream_ptr(params.device))
    _lib.check(rc, "fp8_adamw_expand_step")


def fp8_adamw_step(params, grads, exp_avg, scale_exp_avg, exp_avg_sq, scale_exp_avg_sq,
                   beta1, beta2, lr, wd, eps, step, qgroup_size, *, bf16_out=None, flags=0):
    """qoptim_cuda.fp8_adamw_step (coat/optimizer/kernels/include/fp8_adamw.h:6-14)."""
    if qgroup_size != 128:
        raise RuntimeError("Only Support 128 per-group quantization currently")
    n = params.numel()
    groups = (n + 127) // 128
    _check_state("scale_exp_avg", scale_exp_avg, groups)
    _check_state("scale_exp_avg_sq", scale_exp_avg_sq, groups)
    if grads.dtype != params.dtype or grads.numel() != n:
        raise RuntimeError("grads must match params in dtype and size")
    P = _lib.dev_ptr
    P(params, "params")  # raises for a CPU tensor before any device is selected
    with torch.cuda.device(params.device):
        rc = _lib.lib().coat_fp8_adamw_step(
            P(params, "params"), P(grads, "grads"), P(exp_avg, "exp_avg"), P(scale_exp_avg),
            P(exp_avg_sq, "exp_avg_sq"), P(scale_exp_avg_sq), beta1, beta2, lr, wd, eps, int(step),
            int(qgroup_size), n, _lib.param_dtype(params), P(bf16_out), int(flags),
            _lib.stream_ptr(params.device))
    _lib.check(rc, "fp8_adamw_step")
