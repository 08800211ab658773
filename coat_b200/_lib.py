"""ctypes binding of libcoat_b200.so, the C-ABI library of hand-written sm_100a kernels.

There is no fallback: if the library is missing, or a kernel is asked to run on
anything but a CUDA tensor, the call raises.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("COAT_B200_LIB", os.path.join(_HERE, "libcoat_b200.so"))

F32, BF16, F16 = 0, 1, 2
E4M3, E5M2 = 0, 1
ADAMW_EXACT_POW = 1
MAX_PEERS = 7            # COAT_MAX_PEERS
PEER_HANDLE_BYTES = 64   # COAT_PEER_HANDLE_BYTES
QUANT_IEEE_DIV = 1
QUANT_STOCHASTIC = 2
E_BADARG, E_TOOBIG, E_TIMEOUT = -1, -7, -8   # COAT_E_* codes that callers test for

# Default flags of the quantizer entry points: 0 = the reference's (Triton's) division, QUANT_IEEE_DIV
# = IEEE division.  Tests that compare with the CPU checker switch it.
quant_flags = 0

_lib = None

_c = ctypes
_vp, _f, _i, _i64 = _c.c_void_p, _c.c_float, _c.c_int, _c.c_int64

# name -> argtypes; every function returns int (0 or a negative COAT_E_* code)
SIGNATURES = {
    "coat_check_device": [],
    "coat_fp8_adamw_expand_step": [_vp] * 10 + [_f] * 5 + [_i, _i, _i, _i64, _i, _vp, _i, _vp],
    "coat_fp8_adamw_step": [_vp] * 6 + [_f] * 5 + [_i, _i, _i64, _i, _vp, _i, _vp],
    "coat_fp8_adamw_multi_step": [_vp, _vp, _i, _i64, _i] + [_f] * 5 + [_i, _i, _i, _i, _i, _vp],
    "coat_fp8_adamw_multi_step_bcast": [_vp, _vp, _i, _i64, _i] + [_f] * 5 + [_i, _i, _i, _i, _i, _vp, _i, _vp],
    "coat_peer_buffer_create": [_i64, _vp, _vp],
    "coat_peer_buffer_open": [_vp, _vp],
    "coat_peer_buffer_close": [_vp],
    "coat_peer_buffer_free": [_vp],
    "coat_peer_copy_async": [_vp, _vp, _i64, _vp],
    "coat_fp8_quantize": [_vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_group_scales_amax": [_vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_division": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _i, _i, _vp],
    "coat_fp8_quantize_transpose": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_quantize_pertensor_static": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _i, _i, _vp],
    "coat_rope_bf16": [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i, _vp],
    "coat_rope_bf16_f32tables": [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i, _vp],
    "coat_fp8_gemm_blockscaled": [_vp, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i, _i, _vp],
    "coat_fp8_quantize_block128": [_vp, _i64, _i64, _i64] + [_vp] * 8 + [_i, _i, _i, _i, _vp],
    "coat_fp8_transpose": [_vp, _vp, _i64, _i64, _vp],
    "coat_fp8_dequantize": [_vp, _vp, _vp, _i64, _i64, _i, _i, _i, _vp],
    "coat_fp8_silu_forward": [_vp, _vp, _vp, _vp, _i64, _i64, _i, _i, _i, _i, _vp],
    "coat_fp8_act_backward": [_i, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_gelu_forward": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i, _i, _i, _i, _vp],
    "coat_fp8_mul_forward": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i, _i, _i, _i, _vp],
    "coat_fp8_mul_forward_pertensor": [_vp] * 8 + [_i64, _i64, _i, _i, _i, _i, _vp],
    "coat_fp8_mul_backward": [_vp] * 9 + [_i64, _i64, _i, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_add": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_silu_mul_forward": [_vp] * 9 + [_i64, _i64, _i, _i, _i, _i, _vp],
    "coat_fp8_mul_silu_backward": [_vp] * 13 + [_i64, _i64, _i, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_rmsnorm_forward": [_vp] * 7 + [_i64, _i64, _i, _f, _i, _i, _i, _i, _vp],
    "coat_fp8_rmsnorm_backward": [_vp] * 9 + [_i, _vp, _i64, _i64, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_quantize_pertensor": [_vp] * 6 + [_i64, _i64, _i64, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_quantize_device_status": [],
    "coat_fp8_quantize_set_barrier_limit": [_i],
    "coat_fp8_layernorm_forward": [_vp] * 9 + [_i64, _i64, _i, _f, _i, _i, _i, _i, _vp],
    "coat_fp8_layernorm_backward": [_vp] * 8 + [_i, _vp, _vp, _i64, _i64, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_gemm": [_vp] * 7 + [_i64, _i64, _i64, _i, _i, _i, _i, _i, _i, _i, _vp],
    "coat_fp8_gemm_device_status": [],
    "coat_cross_entropy_inplace": [_vp, _i, _i64, _vp, _vp, _i64, _i64, _i64, _f, _vp],
    "coat_fp8_adamw_debug_counters": [_vp],
    "coat_fp8_adamw_device_status": [],
}


class CoatAdamwTensor(ctypes.Structure):
    """Mirror of `struct CoatAdamwTensor` in include/coat_b200.h."""
    _fields_ = [(n, _vp) for n in ("p", "g", "m", "v", "s_m", "k_m", "r_m", "s_v", "k_v", "r_v", "bf16_out")] + [
        ("numel", _i64)]


def lib():
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m coat_b200.csrc.build` "
                "(there is no non-CUDA fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _i
        L.coat_strerror.argtypes = [_i]
        L.coat_strerror.restype = _c.c_char_p
        L.coat_b200_version.restype = _c.c_char_p
        _lib = L
    return _lib


def check(code, what=""):
    if code != 0:
        msg = lib().coat_strerror(code).decode()
        raise RuntimeError(f"coat_b200 {what}: {msg} (code {code})")


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def dev_ptr(t, name="tensor"):
    """Device address of a contiguous CUDA tensor (None passes through as NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError(f"coat_b200: {name} must be a CUDA tensor (no CPU path exists)")
    if not t.is_contiguous():
        raise RuntimeError(f"coat_b200: {name} must be contiguous")
    return t.data_ptr()


def param_dtype(t):
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float16:
        return F16
    raise RuntimeError(f"coat_b200: unsupported parameter dtype {t.dtype}")


def float_dtype(t_or_dtype):
    dt = t_or_dtype.dtype if isinstance(t_or_dtype, torch.Tensor) else t_or_dtype
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    raise RuntimeError(f"coat_b200: unsupported floating dtype {dt}")


def fp8_enum_of(t):
    if t.dtype == torch.float8_e4m3fn:
        return E4M3
    if t.dtype == torch.float8_e5m2:
        return E5M2
    raise RuntimeError(f"coat_b200: expected an fp8 tensor, got {t.dtype}")


_FP8_NAMES = {"E4M3": (E4M3, torch.float8_e4m3fn), "E5M2": (E5M2, torch.float8_e5m2)}


def fp8_format(fp8type):
    """Accepts "E4M3"/"E5M2" or a torch fp8 dtype, as the reference wrappers do
    (coat/activation/real_quantization/_quantize.py:132-133)."""
    if isinstance(fp8type, str):
        return _FP8_NAMES[fp8type]
    if fp8type == torch.float8_e4m3fn:
        return E4M3, fp8type
    if fp8type == torch.float8_e5m2:
        return E5M2, fp8type
    raise RuntimeError(f"coat_b200: unsupported fp8 type {fp8type}")
