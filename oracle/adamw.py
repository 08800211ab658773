"""ctypes front-end of oracle/fp8_adamw_oracle.c (TEST INFRASTRUCTURE ONLY).

The C file restates coat/optimizer/kernels/fp8_adamw_expand_cuda_kernel.cu:42-202
and coat/optimizer/kernels/fp8_adamw_cuda_kernel.cu:38-124 for the CPU.  All
functions take CPU torch tensors (or numpy arrays) and update them in place, with
the argument order of qoptim_cuda.fp8_adamw_expand_step / fp8_adamw_step
(coat/optimizer/kernels/bindings.cpp:6-7).
"""
import ctypes
import os
import subprocess

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

UNFUSED_P = 1


def build(force=False):
    src = os.path.join(_HERE, "fp8_adamw_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "-B", "_build/liboracle.so"], check=True, capture_output=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        f, i, i64, vp = ctypes.c_float, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p
        _lib.oracle_fp8_adamw_expand_step.argtypes = [vp] * 10 + [f] * 5 + [i, i, i, i64, i, i]
        _lib.oracle_fp8_adamw_expand_step.restype = None
        _lib.oracle_fp8_adamw_step.argtypes = [vp] * 6 + [f] * 5 + [i, i, i64, i, i]
        _lib.oracle_fp8_adamw_step.restype = None
        _lib.oracle_fp8_adamw_dequant.argtypes = [vp] * 5 + [i64, i]
        _lib.oracle_fp8_adamw_dequant.restype = None
        _lib.oracle_encode_fp8.argtypes = [vp, vp, i64, i]
        _lib.oracle_decode_fp8.argtypes = [vp, vp, i64, i]
        _lib.oracle_float_to_bf16.argtypes = [f]
        _lib.oracle_float_to_bf16.restype = ctypes.c_uint16
        _lib.oracle_set_num_threads.argtypes = [i]
        _lib.oracle_set_num_threads.restype = None
        _lib.oracle_max_threads.restype = i
    return _lib


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        assert t.flags["C_CONTIGUOUS"]
        return t.ctypes.data
    assert t.device.type == "cpu" and t.is_contiguous()
    return t.data_ptr()


def _pdtype(p):
    if p.dtype == torch.float32:
        return 0
    if p.dtype == torch.bfloat16:
        return 1
    raise TypeError("oracle supports fp32 and bf16 parameters")


def fp8_adamw_expand_step(p, g, m, s_m, k_m, r_m, v, s_v, k_v, r_v, beta1, beta2, lr, wd, eps, step,
                          qgroup_size, expand_min, flags=0):
    assert qgroup_size == 128, "Only Support 128 per-group quantization currently"
    n = p.numel()
    assert s_m.numel() == (n + 127) // 128 and s_v.numel() == (n + 127) // 128
    for t in (s_m, k_m, r_m, s_v, k_v, r_v):
        assert t.dtype == torch.float32
    lib().oracle_fp8_adamw_expand_step(_ptr(p), _ptr(g), _ptr(m), _ptr(s_m), _ptr(k_m), _ptr(r_m), _ptr(v),
                                       _ptr(s_v), _ptr(k_v), _ptr(r_v), beta1, beta2, lr, wd, eps, int(step),
                                       qgroup_size, expand_min, n, _pdtype(p), flags)


def fp8_adamw_step(p, g, m, s_m, v, s_v, beta1, beta2, lr, wd, eps, step, qgroup_size, flags=0):
    assert qgroup_size == 128, "Only Support 128 per-group quantization currently"
    n = p.numel()
    assert s_m.numel() == (n + 127) // 128 and s_v.numel() == (n + 127) // 128
    lib().oracle_fp8_adamw_step(_ptr(p), _ptr(g), _ptr(m), _ptr(s_m), _ptr(v), _ptr(s_v), beta1, beta2, lr, wd,
                                eps, int(step), qgroup_size, n, _pdtype(p), flags)


def dequant_state(codes, scale, expand=None, sqrtminmax=None, second=False):
    out = torch.empty(codes.numel(), dtype=torch.float32)
    lib().oracle_fp8_adamw_dequant(_ptr(codes), _ptr(scale), _ptr(expand), _ptr(sqrtminmax), _ptr(out),
                                   codes.numel(), int(second))
    return out.view(codes.shape)


def encode_fp8(x, fmt="E4M3"):
    x = x.detach().to(torch.float32).contiguous()
    out = torch.empty(x.shape, dtype=torch.uint8)
    lib().oracle_encode_fp8(_ptr(x), _ptr(out), x.numel(), 0 if fmt == "E4M3" else 1)
    return out


def decode_fp8(c, fmt="E4M3"):
    c = c.contiguous().view(torch.uint8)
    out = torch.empty(c.shape, dtype=torch.float32)
    lib().oracle_decode_fp8(_ptr(c), _ptr(out), c.numel(), 0 if fmt == "E4M3" else 1)
    return out


def set_num_threads(n):
    """Use `n` OpenMP threads in the step functions, whatever OMP_NUM_THREADS says; returns the count in effect."""
    lib().oracle_set_num_threads(int(n))
    return int(lib().oracle_max_threads())
