"""Host side of the quantizers: same names, positional arguments and return tuples as the reference's
python wrappers; each allocates its outputs with torch and makes one or two calls into the C ABI.

Reference wrappers mirrored here:
  fp8_quantize                      _quantize.py:120-163
  fp8_quantize_pertensor            _quantize_pertensor.py:106-147
  fp8_quantize_pertensor_transpose  _quantize_pertensor_transpose.py:106-150
  fp8_division                      _division.py:153-207
  fp8_division_transpose            _division_transpose.py:147-210
  fp8_quantize_transpose            _quantize_transpose.py:176-226
  fp8_transpose                     _transpose.py:85-115
  fp8_dequantize                    _dequantize.py:119-156
(paths under coat/activation/real_quantization/).
"""
import os

import torch

from ... import _lib
from .common import FP8_MAX_VALUE, SCALE_MIN_THRES, convert_str_to_fp8


def _flat2d(x):
    """3-D inputs are treated as (B*S, H), as the reference does."""
    if x.dim() == 3:
        return x.reshape(-1, x.shape[-1]), x.shape[0]
    if x.dim() != 2:
        raise RuntimeError(f"expected a 2-D or 3-D tensor, got {x.dim()}-D")
    return x, None


def _fp8_dtype(fp8type):
    if isinstance(fp8type, str):
        return convert_str_to_fp8[fp8type]
    return fp8type


def _prep(x):
    x, bs = _flat2d(x)
    if not x.is_cuda:
        raise RuntimeError("coat_b200: the quantizers need CUDA tensors (no CPU path exists)")
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x, bs


def _call(name, *args):
    _lib.check(getattr(_lib.lib(), name)(*args), name)


def _flags(flags):
    return _lib.quant_flags if flags is None else flags


def fp8_quantize(x, QB, fp8type, scale_dtype=torch.bfloat16, *, flags=None):
    x, bs = _prep(x)
    M, N = x.shape
    fp8type = _fp8_dtype(fp8type)
    y = torch.empty((M, N), dtype=fp8type, device=x.device)
    s_y = torch.empty((M, N // QB), dtype=scale_dtype, device=x.device)
    with torch.cuda.device(x.device):
        _call("coat_fp8_quantize", x.data_ptr(), y.data_ptr(), s_y.data_ptr(), M, N, x.stride(0), QB,
              _lib.fp8_enum_of(y), _lib.float_dtype(x), _lib.float_dtype(scale_dtype), _flags(flags),
              _lib.stream_ptr(x.device))
    if bs is not None:
        y = y.reshape(bs, -1, y.shape[-1])
        s_y = s_y.reshape(bs, -1, s_y.shape[-1])
    return y, s_y


def _flags_stochastic(flags, stochastic):
    """Division flags with the reference's stochastic rounding (_division.py:96-150) switched on or not."""
    return _flags(flags) | (_lib.QUANT_STOCHASTIC if stochastic else 0)


_SYNC_WORDS = {}
# COAT_PERTENSOR_ONE_LAUNCH=0: always take the two-call form (a cooperative launch needs every SM the library counts;
# on a GPU partitioned by MPS limits or green contexts it is refused with a launch error)
_ONE_LAUNCH = os.environ.get("COAT_PERTENSOR_ONE_LAUNCH", "1") != "0"


def _sync_words(dev):
    """Three zero words per (device, stream) for the one-launch per-tensor kernel, which needs them zero on entry
    and leaves them zero (allocated and cleared once; calls ordered on a stream share them)."""
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), _lib.stream_ptr(dev))
    if torch.cuda.is_current_stream_capturing():
        # memory allocated during a capture belongs to the graph's pool: use fresh words (their memset is captured)
        return None, torch.zeros(4, dtype=torch.int32, device=dev)
    words = _SYNC_WORDS.get(key)
    if words is None:
        words = _SYNC_WORDS[key] = torch.zeros(4, dtype=torch.int32, device=dev)
    return key, words


def _pertensor(x, QB, fp8type, scale_dtype, want_scales, want_straight, want_transposed, flags, stochastic=False):
    """Per-tensor quantize.  Normally one cooperative launch that re-reads x from L2; with stochastic rounding, or
    a transposed copy of a matrix whose row count is not a multiple of 16, pass 1 (tensor amax, optional group
    scales) + pass 2 (division by the one scale, straight and / or transposed)."""
    M, N = x.shape
    fmt = _lib.fp8_format(fp8type)[0]
    dev = x.device
    sync = torch.empty(1, dtype=torch.int32, device=dev)   # amax word of the two-call form, zeroed by pass 1
    s_y = torch.empty((M, N // QB), dtype=scale_dtype, device=dev) if want_scales else None
    s_max = torch.empty((), dtype=scale_dtype, device=dev)
    y = torch.empty((M, N), dtype=fp8type, device=dev) if want_straight else None
    y_t = torch.empty((N, M), dtype=fp8type, device=dev) if want_transposed else None
    P = lambda t: None if t is None else t.data_ptr()
    with torch.cuda.device(dev):
        st = _lib.stream_ptr(dev)
        # the transposing form of the one-launch kernel walks 128 x 128 tiles: no group scales, M % 16 == 0
        one_launch = (_ONE_LAUNCH and not stochastic and
                      (not want_transposed or (not want_scales and M % 16 == 0)))
        if one_launch:
            key, words = _sync_words(dev)
            try:
                _call("coat_fp8_quantize_pertensor", x.data_ptr(), P(y), P(y_t), P(s_y), s_max.data_ptr(),
                      words.data_ptr(), M, N, x.stride(0), QB, fmt, _lib.float_dtype(x), _lib.float_dtype(scale_dtype),
                      _flags(flags), st)
            except Exception:
                _SYNC_WORDS.pop(key, None)   # do not reuse words a failed call may have left dirty
                raise
            return y, s_max, s_y, y_t
        _call("coat_fp8_group_scales_amax", x.data_ptr(), P(s_y), sync.data_ptr(), M, N, x.stride(0), QB, fmt,
              _lib.float_dtype(x), _lib.float_dtype(scale_dtype), _flags(flags), st)
        _call("coat_fp8_division", x.data_ptr(), P(y), P(y_t), None, s_max.data_ptr(), sync.data_ptr(), M, N,
              x.stride(0), fmt, _lib.float_dtype(x), _lib.float_dtype(scale_dtype), _flags_stochastic(flags, stochastic),
              st)
    return y, s_max, s_y, y_t


def fp8_quantize_pertensor(x, QB, fp8type, stochastic=False, scale_dtype=torch.bfloat16, *, flags=None):
    x, bs = _prep(x)
    fp8type = _fp8_dtype(fp8type)
    y, s_max, s_y, _ = _pertensor(x, QB, fp8type, scale_dtype, True, True, False, flags, stochastic)
    if bs is not None:
        y = y.reshape(bs, -1, y.shape[-1])
        s_y = s_y.reshape(bs, -1, s_y.shape[-1])
    return y, s_max, s_y


def fp8_quantize_pertensor_transpose(x, QB, fp8type, transpose_output_2d=False, stochastic=False,
                                     scale_dtype=torch.bfloat16, *, flags=None):
    x, bs = _prep(x)
    fp8type = _fp8_dtype(fp8type)
    qy, s_max, _, qy_t = _pertensor(x, QB, fp8type, scale_dtype, False, True, True, flags, stochastic)
    if bs is not None:
        qy = qy.reshape(bs, -1, qy.shape[-1])
        if not transpose_output_2d:
            qy_t = qy_t.reshape(bs, -1, qy_t.shape[-1])
    return qy, s_max, qy_t


def _default_scale(x, fp8type, flags):
    """(x.abs().max() + 1e-10) / fp8_max in x's dtype, the reference's default when no scale is passed
    (_division.py:178-179); the maximum comes from the amax kernel, the two scalar operations are torch's."""
    M, N = x.shape
    amax = torch.empty(1, dtype=torch.int32, device=x.device)
    with torch.cuda.device(x.device):
        _call("coat_fp8_group_scales_amax", x.data_ptr(), None, amax.data_ptr(), M, N, x.stride(0), 16,
              _lib.fp8_format(fp8type)[0], _lib.float_dtype(x), _lib.BF16, _flags(flags), _lib.stream_ptr(x.device))
    return (amax.view(torch.float32)[0].to(x.dtype) + SCALE_MIN_THRES) / FP8_MAX_VALUE[fp8type]


def fp8_pertensor_scale(x, fp8type, *, flags=None):
    """The per-tensor scale alone, (x.abs().max() + 1e-10) / fp8_max in x's dtype: what `fp8_division(x, QB, fp8type)`
    returns as its scale when none is passed (_division.py:178-179), without quantising anything.  For callers
    that keep only the scale (the weight cache in memory-efficient mode)."""
    x, _ = _prep(x)
    return _default_scale(x, _fp8_dtype(fp8type), flags)


def _division(x, fp8type, s_y, want_straight, want_transposed, flags, stochastic=False):
    M, N = x.shape
    want_straight = want_straight or stochastic   # the stochastic transposed copy is made from the straight one
    if s_y is None:
        s_y = _default_scale(x, fp8type, flags)
    if not torch.is_tensor(s_y):
        s_y = torch.tensor(float(s_y), dtype=torch.float32, device=x.device)
    if not s_y.is_cuda:
        s_y = s_y.to(x.device)
    y = torch.empty((M, N), dtype=fp8type, device=x.device) if want_straight else None
    y_t = torch.empty((N, M), dtype=fp8type, device=x.device) if want_transposed else None
    P = lambda t: None if t is None else t.data_ptr()
    with torch.cuda.device(x.device):
        _call("coat_fp8_division", x.data_ptr(), P(y), P(y_t), s_y.data_ptr(), None, None, M, N, x.stride(0),
              _lib.fp8_format(fp8type)[0], _lib.float_dtype(x), _lib.float_dtype(s_y),
              _flags_stochastic(flags, stochastic), _lib.stream_ptr(x.device))
    return y, s_y, y_t


def fp8_division(x, QB, fp8type, s_y=None, stochastic=False, *, flags=None):
    x, bs = _prep(x)
    fp8type = _fp8_dtype(fp8type)
    y, s_y, _ = _division(x, fp8type, s_y, True, False, flags, stochastic)
    if bs is not None:
        y = y.reshape(bs, -1, y.shape[-1])
    return y, s_y


def fp8_division_transpose(x, QB, fp8type, s_y=None, stochastic=False, only_transposed=False, *, flags=None):
    x, bs = _prep(x)
    fp8type = _fp8_dtype(fp8type)
    y, s_y, y_t = _division(x, fp8type, s_y, not only_transposed, True, flags, stochastic)
    if only_transposed:
        return y_t, s_y
    if bs is not None:
        y = y.reshape(bs, -1, y.shape[-1])
    return y, s_y, y_t   # y_t stays 2-D


def _block128(x, fp8type, scale_dtype, flags, block=False, block_t=False, rows=False, cols_t=False):
    """One call of coat_fp8_quantize_block128; returns the four (codes, scales) pairs, None where not asked for."""
    M, N = x.shape
    dev = x.device

    def pair(want, shape, sshape):
        if not want:
            return None, None
        return torch.empty(shape, dtype=fp8type, device=dev), torch.empty(sshape, dtype=scale_dtype, device=dev)

    y_b, s_b = pair(block, (M, N), (M // 128, N // 128))
    y_bt, s_bt = pair(block_t, (N, M), (N // 128, M // 128))
    y_r, s_r = pair(rows, (M, N), (M, N // 128))
    y_ct, s_ct = pair(cols_t, (N, M), (N, M // 128))
    ptr = lambda t: None if t is None else t.data_ptr()
    with torch.cuda.device(dev):
        _call("coat_fp8_quantize_block128", x.data_ptr(), M, N, x.stride(0), ptr(y_b), ptr(s_b), ptr(y_bt), ptr(s_bt),
              ptr(y_r), ptr(s_r), ptr(y_ct), ptr(s_ct), _lib.fp8_format(fp8type)[0], _lib.float_dtype(x),
              _lib.float_dtype(scale_dtype), _flags(flags), _lib.stream_ptr(dev))
    return (y_b, s_b), (y_bt, s_bt), (y_r, s_r), (y_ct, s_ct)


def fp8_quantize_perblock(x, QB, fp8type, scale_dtype=torch.bfloat16, *, flags=None):
    """One scale per QB x QB block, QB = 128 (_quantize_perblock.py:115-150).  -> (y, s_y[M/QB, N/QB]), 2-D."""
    if QB != 128:
        raise RuntimeError("coat_b200: per-block quantization is provided for QB = 128")
    x, _ = _prep(x)
    return _block128(x, _fp8_dtype(fp8type), scale_dtype, flags, block=True)[0]


def fp8_quantize_perblock_transpose(x, QB, fp8type, scale_dtype=torch.bfloat16, only_transposed=False, *, flags=None):
    """-> (y, s_y), (y_t, s_y_t), or only the transposed pair (_quantize_perblock_transpose.py:127-190)."""
    if QB != 128:
        raise RuntimeError("coat_b200: per-block quantization is provided for QB = 128")
    x, _ = _prep(x)
    out = _block128(x, _fp8_dtype(fp8type), scale_dtype, flags, block=not only_transposed, block_t=True)
    return out[1] if only_transposed else (out[0], out[1])


def fp8_quantize_perblock_transpose_pergroup(x, QB, fp8type, scale_dtype=torch.bfloat16, only_transposed=False, *,
                                             flags=None):
    """-> (y, s_y), (y_t, s_y_t), (y_pg, s_y_pg): block-scaled codes, their transpose, and 1 x QB row-group codes
    (_quantize_perblock_transpose_pergroup.py:183-246).  With only_transposed the first pair is not computed
    (the reference returns uninitialised buffers there); None is returned in its place."""
    if QB != 128:
        raise RuntimeError("coat_b200: per-block quantization is provided for QB = 128")
    x, _ = _prep(x)
    out = _block128(x, _fp8_dtype(fp8type), scale_dtype, flags, block=not only_transposed, block_t=True, rows=True)
    return out[0], out[1], out[2]


def fp8_quantize_transpose(x, QB, fp8type, scale_dtype=torch.bfloat16, *, flags=None):
    x, _ = _prep(x)
    M, N = x.shape
    fp8type = _fp8_dtype(fp8type)
    if QB == 128:
        out = _block128(x, fp8type, scale_dtype, flags, rows=True, cols_t=True)
        return out[2], out[3]
    y = torch.empty((M, N), dtype=fp8type, device=x.device)
    y_t = torch.empty((N, M), dtype=fp8type, device=x.device)
    s_y = torch.empty((M, N // QB), dtype=scale_dtype, device=x.device)
    s_y_t = torch.empty((N, M // QB), dtype=scale_dtype, device=x.device)
    with torch.cuda.device(x.device):
        _call("coat_fp8_quantize_transpose", x.data_ptr(), y.data_ptr(), s_y.data_ptr(), y_t.data_ptr(),
              s_y_t.data_ptr(), M, N, x.stride(0), QB, _lib.fp8_enum_of(y), _lib.float_dtype(x),
              _lib.float_dtype(scale_dtype), _flags(flags), _lib.stream_ptr(x.device))
    return (y, s_y), (y_t, s_y_t)


def fp8_transpose(x, transpose_output_2d=False):
    x, bs = _flat2d(x)
    if not x.is_cuda:
        raise RuntimeError("coat_b200: fp8_transpose needs a CUDA tensor")
    x = x.contiguous()
    M, N = x.shape
    y = torch.empty((N, M), dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        _call("coat_fp8_transpose", x.data_ptr(), y.data_ptr(), M, N, _lib.stream_ptr(x.device))
    if bs is not None and not transpose_output_2d:
        y = y.reshape(bs, -1, y.shape[-1])
    return y


def fp8_dequantize(x, s_x, QB):
    x, bs = _flat2d(x)
    if not x.is_cuda:
        raise RuntimeError("coat_b200: fp8_dequantize needs CUDA tensors")
    x = x.contiguous()
    s_x = s_x.reshape(-1, s_x.shape[-1]).contiguous()
    M, N = x.shape
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        _call("coat_fp8_dequantize", x.data_ptr(), s_x.data_ptr(), y.data_ptr(), M, N, QB, _lib.fp8_enum_of(x),
              _lib.float_dtype(s_x), _lib.stream_ptr(x.device))
    if bs is not None:
        y = y.reshape(bs, -1, y.shape[-1])
    return y
