"""Host side of the fused quantize-on-save operators: the reference's names, positional arguments
and return tuples; torch allocates the outputs, the C ABI does the work.

Reference wrappers mirrored (paths under coat/activation/real_quantization/):
  fp8_silu_forward   silu_fwd.py:152-198      fp8_silu_backward  silu_bwd.py:170-238
  fp8_gelu_forward   gelu_fwd.py:152-203      fp8_gelu_backward  gelu_bwd.py:173-230
  fp8_mul_forward    mul_fwd.py:191-254       fp8_mul_backward   mul_bwd.py:221-315
  fp8_add_Ifp_Ifp_Ofp_Og16  add_fwd.py:162-213    fp8_add_Ifp_Ifp_Ofp_Opt  add_bwd.py:147-200
  fp8_rmsnorm_forward / fp8_rmsnorm_backward  func_rmsnorm.py:223-335
Where the reference runs kernel -> `s_y.max()` -> fp8_division[_transpose], the producing kernel here also
leaves the tensor's amax in a 4-byte word and the division derives the same scale from it.
"""
import torch

from ... import _lib
from . import _ops
from ._ops import _call, _flags, _fp8_dtype


def _flat(*ts):
    """Flatten 3-D tensors to 2-D the way the reference does; returns the batch size or None."""
    bs = ts[0].shape[0] if ts[0].dim() == 3 else None
    out = []
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("coat_b200: the fused operators need CUDA tensors (no CPU path exists)")
        out.append(t.reshape(-1, t.shape[-1]).contiguous())
    return out, bs


def _unflat(t, bs):
    return t if bs is None or t is None else t.reshape(bs, -1, t.shape[-1])


def _amax_word(device):
    return torch.empty(1, dtype=torch.int32, device=device)


def _divide(y_bf16, fp8type, amax, want_transposed, flags, scale_dtype=torch.bfloat16, stochastic=False):
    """Per-tensor quantize of a bf16 (LayerNorm: fp32) intermediate with the scale derived from the amax word."""
    M, N = y_bf16.shape
    dev = y_bf16.device
    q = torch.empty((M, N), dtype=fp8type, device=dev)
    q_t = torch.empty((N, M), dtype=fp8type, device=dev) if want_transposed else None
    s_max = torch.empty((), dtype=scale_dtype, device=dev)
    _call("coat_fp8_division", y_bf16.data_ptr(), q.data_ptr(), None if q_t is None else q_t.data_ptr(), None,
          s_max.data_ptr(), amax.data_ptr(), M, N, N, _lib.fp8_format(fp8type)[0], _lib.float_dtype(y_bf16),
          _lib.float_dtype(scale_dtype), _flags(flags) | (_lib.QUANT_STOCHASTIC if stochastic else 0),
          _lib.stream_ptr(dev))
    return q, s_max, q_t


def fp8_silu_forward(x, s_x, QB, *, flags=None):
    (x2, s2), bs = _flat(x, s_x)
    M, N = x2.shape
    y = torch.empty_like(x2)
    s_y = torch.empty_like(s2)
    with torch.cuda.device(x.device):
        _call("coat_fp8_silu_forward", x2.data_ptr(), s2.data_ptr(), y.data_ptr(), s_y.data_ptr(), M, N, QB,
              _lib.fp8_enum_of(x2), _lib.float_dtype(s2), _flags(flags), _lib.stream_ptr(x.device))
    return _unflat(y, bs), _unflat(s_y, bs)


def _act_backward(gelu, x, s_x, g, QB, fp8type, flags):
    (x2, s2, g2), bs = _flat(x, s_x, g)
    M, N = x2.shape
    fp8type = _fp8_dtype(fp8type)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    s_y = torch.empty(s2.shape, dtype=torch.bfloat16, device=x.device)
    amax = _amax_word(x.device)
    _call("coat_fp8_act_backward", int(gelu), x2.data_ptr(), s2.data_ptr(), g2.data_ptr(), y.data_ptr(),
          s_y.data_ptr(), amax.data_ptr(), M, N, QB, _lib.fp8_enum_of(x2), _lib.float_dtype(s2),
          _lib.float_dtype(g2), _lib.fp8_format(fp8type)[0], _flags(flags), _lib.stream_ptr(x.device))
    return y, s_y, amax, bs, fp8type


def fp8_silu_backward(x, s_x, g, QB, fp8type, stochastic=False, output_quantized_transpose=False, *, flags=None):
    # `stochastic` is accepted and has no effect, as in the reference (silu_bwd.py:170-238 never reads it)
    with torch.cuda.device(x.device):
        y, s_y, amax, bs, fp8type = _act_backward(False, x, s_x, g, QB, fp8type, flags)
        if not output_quantized_transpose:
            return _unflat(y, bs), _unflat(s_y, bs)
        qy, s_max, qy_t = _divide(y, fp8type, amax, True, flags)
    return _unflat(qy, bs), s_max, qy_t


def fp8_gelu_forward(x, s_x, QB, transpose_output_2d=False, *, flags=None):
    (x2, s2), bs = _flat(x, s_x)
    M, N = x2.shape
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    s_y = torch.empty_like(s2)
    amax = _amax_word(x.device)
    with torch.cuda.device(x.device):
        _call("coat_fp8_gelu_forward", x2.data_ptr(), s2.data_ptr(), y.data_ptr(), s_y.data_ptr(), amax.data_ptr(),
              M, N, QB, _lib.fp8_enum_of(x2), _lib.float_dtype(s2), _flags(flags), _lib.stream_ptr(x.device))
        qy, s_max, qy_t = _divide(y, x2.dtype, amax, True, flags, scale_dtype=s2.dtype)
    if bs is not None and not transpose_output_2d:
        qy_t = qy_t.reshape(bs, -1, N)
    return _unflat(qy, bs), s_max, qy_t


def fp8_gelu_backward(x, s_x, g, QB, fp8type, *, flags=None):
    with torch.cuda.device(x.device):
        y, s_y, amax, bs, fp8type = _act_backward(True, x, s_x, g, QB, fp8type, flags)
        qy, s_max, _ = _divide(y, fp8type, amax, False, flags)
    return _unflat(qy, bs), s_max


def fp8_mul_forward(x1, s_x1, x2, s_x2, QB, transpose_output_2d=False, *, flags=None):
    (a, sa, b, sb), bs = _flat(x1, s_x1, x2, s_x2)
    assert a.shape == b.shape and sa.shape == sb.shape
    M, N = a.shape
    if (_ops._ONE_LAUNCH and QB == 16 and M % 16 == 0 and N % 128 == 0 and sa.dtype == torch.bfloat16 and
            sb.dtype == torch.bfloat16 and a.dtype == b.dtype):
        # one cooperative launch that recomputes the product in its second pass: no bf16 tensor goes to memory
        dev = a.device
        qy = torch.empty((M, N), dtype=b.dtype, device=dev)
        qy_t = torch.empty((N, M), dtype=b.dtype, device=dev)
        s_max = torch.empty((), dtype=sa.dtype, device=dev)
        with torch.cuda.device(dev):
            key, words = _ops._sync_words(dev)
            try:
                _call("coat_fp8_mul_forward_pertensor", a.data_ptr(), sa.data_ptr(), b.data_ptr(), sb.data_ptr(),
                      qy.data_ptr(), qy_t.data_ptr(), s_max.data_ptr(), words.data_ptr(), M, N, QB, _lib.fp8_enum_of(a),
                      _lib.float_dtype(sa), _flags(flags), _lib.stream_ptr(dev))
            except Exception:
                _ops._SYNC_WORDS.pop(key, None)   # do not reuse words a failed call may have left dirty
                raise
        if bs is not None and not transpose_output_2d:
            qy_t = qy_t.reshape(bs, -1, qy.shape[-1])
        return _unflat(qy, bs), s_max, qy_t
    y = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    s_y = torch.empty_like(sa)
    amax = _amax_word(a.device)
    with torch.cuda.device(a.device):
        _call("coat_fp8_mul_forward", a.data_ptr(), sa.data_ptr(), b.data_ptr(), sb.data_ptr(), y.data_ptr(),
              s_y.data_ptr(), amax.data_ptr(), M, N, QB, _lib.fp8_enum_of(a), _lib.float_dtype(sa), _flags(flags),
              _lib.stream_ptr(a.device))
        qy, s_max, qy_t = _divide(y, b.dtype, amax, True, flags, scale_dtype=sa.dtype)
    if bs is not None and not transpose_output_2d:
        qy_t = qy_t.reshape(bs, -1, qy.shape[-1])
    return _unflat(qy, bs), s_max, qy_t


def fp8_mul_backward(x1, s_x1, x2, s_x2, g, QB, fp8type, stochastic=False, output_quantized_transpose=False, *,
                     flags=None):
    # `stochastic` is accepted and has no effect on the results, as in the reference (mul_bwd.py:236-290 draws
    # a noise tensor and hands the kernel a flag that the kernel never reads)
    (a, sa, b, sb, g2), bs = _flat(x1, s_x1, x2, s_x2, g)
    assert a.shape == b.shape and sa.shape == sb.shape
    M, N = a.shape
    fp8type = _fp8_dtype(fp8type)
    dev = a.device
    y1 = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    y2 = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    s_y2 = torch.empty(sa.shape, dtype=torch.bfloat16, device=dev)
    amax = _amax_word(dev)
    with torch.cuda.device(dev):
        _call("coat_fp8_mul_backward", a.data_ptr(), sa.data_ptr(), b.data_ptr(), sb.data_ptr(), g2.data_ptr(),
              y1.data_ptr(), y2.data_ptr(), s_y2.data_ptr(), amax.data_ptr(), M, N, QB, _lib.fp8_enum_of(a),
              _lib.float_dtype(sa), _lib.float_dtype(g2), _lib.fp8_format(fp8type)[0], _flags(flags),
              _lib.stream_ptr(dev))
        if not output_quantized_transpose:
            return _unflat(y1, bs), (_unflat(y2, bs), _unflat(s_y2, bs))
        qy2, s_max, qy2_t = _divide(y2, fp8type, amax, True, flags)
    return _unflat(y1, bs), (_unflat(qy2, bs), s_max, qy2_t)


def fp8_silu_mul_forward(gate_x, gate_s, up_x, up_s, QB, transpose_output_2d=False, *, flags=None):
    """Forward of `silu(gate) * up` in one elementwise kernel (no counterpart in the reference, which calls
    fp8_silu_forward and fp8_mul_forward one after the other; same bits):
        (silu_x, silu_s), (mul_x, s_max, mul_x_t) = fp8_silu_forward(gate_x, gate_s, QB) and
        fp8_mul_forward(silu_x, silu_s, up_x, up_s, QB, transpose_output_2d)."""
    (a, sa, b, sb), bs = _flat(gate_x, gate_s, up_x, up_s)
    assert a.shape == b.shape and sa.shape == sb.shape and a.dtype == b.dtype and sa.dtype == sb.dtype
    M, N = a.shape
    dev = a.device
    q_silu = torch.empty_like(a)
    s_silu = torch.empty_like(sa)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    amax = _amax_word(dev)
    with torch.cuda.device(dev):
        _call("coat_fp8_silu_mul_forward", a.data_ptr(), sa.data_ptr(), b.data_ptr(), sb.data_ptr(), q_silu.data_ptr(),
              s_silu.data_ptr(), y.data_ptr(), None, amax.data_ptr(), M, N, QB, _lib.fp8_enum_of(a),
              _lib.float_dtype(sa), _flags(flags), _lib.stream_ptr(dev))
        qy, s_max, qy_t = _divide(y, b.dtype, amax, True, flags, scale_dtype=sa.dtype)
    if bs is not None and not transpose_output_2d:
        qy_t = qy_t.reshape(bs, -1, qy.shape[-1])
    return (_unflat(q_silu, bs), _unflat(s_silu, bs)), (_unflat(qy, bs), s_max, qy_t)


def fp8_mul_silu_backward(silu_x, silu_s, up_x, up_s, gate_x, gate_s, g, QB, fp8type, *, flags=None):
    """Backward of `silu(gate) * up` in one elementwise kernel (no counterpart in the reference, which calls
    fp8_mul_backward and fp8_silu_backward one after the other; same bits):
        (d_up, s, d_up_t), (d_gate, s, d_gate_t) = per-tensor FP8 codes, scale and transposed codes of the
        gradients towards the up and the gate projections, i.e.
        fp8_mul_backward(silu_x, silu_s, up_x, up_s, g, QB, fp8type, output_quantized_transpose=True)[1] and
        fp8_silu_backward(gate_x, gate_s, <first output of that call>, QB, fp8type, output_quantized_transpose=True)."""
    (a, sa, b, sb, c, sc, g2), bs = _flat(silu_x, silu_s, up_x, up_s, gate_x, gate_s, g)
    assert a.shape == b.shape == c.shape == g2.shape and sa.shape == sb.shape == sc.shape
    assert a.dtype == b.dtype == c.dtype and sa.dtype == sb.dtype == sc.dtype
    M, N = a.shape
    fp8type = _fp8_dtype(fp8type)
    dev = a.device
    y_up = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    y_gate = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    s_up = torch.empty(sa.shape, dtype=torch.bfloat16, device=dev)
    s_gate = torch.empty(sa.shape, dtype=torch.bfloat16, device=dev)
    amax_up, amax_gate = _amax_word(dev), _amax_word(dev)
    with torch.cuda.device(dev):
        _call("coat_fp8_mul_silu_backward", a.data_ptr(), sa.data_ptr(), b.data_ptr(), sb.data_ptr(), c.data_ptr(),
              sc.data_ptr(), g2.data_ptr(), y_up.data_ptr(), s_up.data_ptr(), amax_up.data_ptr(), y_gate.data_ptr(),
              s_gate.data_ptr(), amax_gate.data_ptr(), M, N, QB, _lib.fp8_enum_of(a), _lib.float_dtype(sa),
              _lib.float_dtype(g2), _lib.fp8_format(fp8type)[0], _flags(flags), _lib.stream_ptr(dev))
        q_up, smax_up, q_up_t = _divide(y_up, fp8type, amax_up, True, flags)
        q_gate, smax_gate, q_gate_t = _divide(y_gate, fp8type, amax_gate, True, flags)
    return (_unflat(q_up, bs), smax_up, q_up_t), (_unflat(q_gate, bs), smax_gate, q_gate_t)


def fp8_mul_silu_backward_joint(silu_x, silu_s, up_x, up_s, gate_x, gate_s, g, QB, fp8type, *, flags=None):
    """Backward of `silu(gate) * up` when the up and gate projections are ONE fused linear layer (the OLMo block,
    coat/models/coat_olmo.py:596-611 of the reference): the gradients d_up and d_gate are concatenated along the last
    dimension and quantised per tensor with the larger of their two scales,
        fp8_division_transpose(cat([d_up, d_gate], -1), QB, fp8type, max(cat([s_up_groups, s_gate_groups])))
    with d_up, d_gate and the group scales as fp8_mul_backward and fp8_silu_backward return them.  Returns
    (codes [M, 2N], scale, transposed codes [2N, M]); same bits.  One elementwise kernel leaves both bf16 gradients
    and their common amax; two division passes write the transposed codes straight into the halves of the joint
    buffer, and only the one-byte codes are concatenated."""
    (a, sa, b, sb, c, sc, g2), bs = _flat(silu_x, silu_s, up_x, up_s, gate_x, gate_s, g)
    assert a.shape == b.shape == c.shape == g2.shape and sa.shape == sb.shape == sc.shape
    assert a.dtype == b.dtype == c.dtype and sa.dtype == sb.dtype == sc.dtype
    M, N = a.shape
    fp8type = _fp8_dtype(fp8type)
    dev = a.device
    y_up = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    y_gate = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    s_up = torch.empty(sa.shape, dtype=torch.bfloat16, device=dev)
    s_gate = torch.empty(sa.shape, dtype=torch.bfloat16, device=dev)
    amax = _amax_word(dev)   # one word for both gradients: the maximum over the concatenation
    q_up = torch.empty((M, N), dtype=fp8type, device=dev)
    q_gate = torch.empty((M, N), dtype=fp8type, device=dev)
    q_t = torch.empty((2 * N, M), dtype=fp8type, device=dev)
    s_max = torch.empty((), dtype=torch.bfloat16, device=dev)
    fmt = _lib.fp8_format(fp8type)[0]
    with torch.cuda.device(dev):
        _call("coat_fp8_mul_silu_backward", a.data_ptr(), sa.data_ptr(), b.data_ptr(), sb.data_ptr(), c.data_ptr(),
              sc.data_ptr(), g2.data_ptr(), y_up.data_ptr(), s_up.data_ptr(), amax.data_ptr(), y_gate.data_ptr(),
              s_gate.data_ptr(), amax.data_ptr(), M, N, QB, _lib.fp8_enum_of(a), _lib.float_dtype(sa),
              _lib.float_dtype(g2), fmt, _flags(flags), _lib.stream_ptr(dev))
        for y, q, rows in ((y_up, q_up, q_t[:N]), (y_gate, q_gate, q_t[N:])):
            _call("coat_fp8_division", y.data_ptr(), q.data_ptr(), rows.data_ptr(), None, s_max.data_ptr(),
                  amax.data_ptr(), M, N, N, fmt, _lib.float_dtype(y), _lib.float_dtype(torch.bfloat16), _flags(flags),
                  _lib.stream_ptr(dev))
    return _unflat(torch.cat((q_up, q_gate), dim=-1), bs), s_max, q_t


def _add(x1, x2, QB, fp8type, want_codes, want_amax, flags):
    (a, b), bs = _flat(x1, x2)
    assert a.shape == b.shape
    M, N = a.shape
    dev = a.device
    y1 = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    y2 = torch.empty((M, N), dtype=fp8type, device=dev) if want_codes else None
    s_y2 = torch.empty((M, N // QB), dtype=torch.bfloat16, device=dev)
    amax = _amax_word(dev) if want_amax else None
    _call("coat_fp8_add", a.data_ptr(), b.data_ptr(), y1.data_ptr(), None if y2 is None else y2.data_ptr(),
          s_y2.data_ptr(), None if amax is None else amax.data_ptr(), M, N, QB, _lib.float_dtype(a),
          _lib.float_dtype(b), _lib.fp8_format(fp8type)[0], _flags(flags), _lib.stream_ptr(dev))
    return y1, y2, s_y2, amax, bs


def fp8_add_Ifp_Ifp_Ofp_Og16(x1, x2, fp8type, QB, *, flags=None):
    fp8type = _fp8_dtype(fp8type)
    with torch.cuda.device(x1.device):
        y1, y2, s_y2, _, bs = _add(x1, x2, QB, fp8type, True, False, flags)
    return _unflat(y1, bs), (_unflat(y2, bs), _unflat(s_y2, bs))


def fp8_add_Ifp_Ifp_Ofp_Opt(x1, x2, QB, fp8type, stochastic=False, *, flags=None):
    fp8type = _fp8_dtype(fp8type)
    with torch.cuda.device(x1.device):
        y1, _, s_y2, amax, bs = _add(x1, x2, QB, fp8type, False, True, flags)
        qy2, s_max, _ = _divide(y1, fp8type, amax, False, flags, stochastic=stochastic)   # add_bwd.py:192
    return _unflat(y1, bs), (_unflat(qy2, bs), s_max, _unflat(s_y2, bs))


def fp8_rmsnorm_forward(x, s_x, w, QB, eps, transpose_output_2d=False, *, flags=None):
    (x2, s2), bs = _flat(x, s_x)
    M, N = x2.shape
    dev = x.device
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    s_y = torch.empty((M,), dtype=torch.bfloat16, device=dev)
    rstd = torch.empty((M,), dtype=torch.float32, device=dev)
    amax = _amax_word(dev)
    w = w.contiguous()
    with torch.cuda.device(dev):
        _call("coat_fp8_rmsnorm_forward", x2.data_ptr(), s2.data_ptr(), w.data_ptr(), y.data_ptr(), s_y.data_ptr(),
              rstd.data_ptr(), amax.data_ptr(), M, N, QB, float(eps), _lib.fp8_enum_of(x2), _lib.float_dtype(s2),
              _lib.float_dtype(w), _flags(flags), _lib.stream_ptr(dev))
        qy, s_max, qy_t = _divide(y, x2.dtype, amax, True, flags)
    if bs is not None and not transpose_output_2d:
        qy_t = qy_t.reshape(bs, -1, N)
    num_warps = 8   # kept in the returned context for signature compatibility; unused here
    return _unflat(qy, bs), s_max, qy_t, (w, rstd, num_warps)


def fp8_rmsnorm_backward(x, s_x, g, w, v, QB, num_warps, *, more_g=()):
    """`more_g`: up to two further bf16 addends of the upstream gradient; the result is that of calling with
    `g + more_g[0] + more_g[1]` (bf16 sums, left to right), without the add kernels."""
    more = [t.reshape(-1, t.shape[-1]) for t in more_g]
    assert len(more) <= 2 and all(t.dtype == torch.bfloat16 and t.is_contiguous() for t in more)
    (x2, s2, g2), bs = _flat(x, s_x, g)
    M, N = g2.shape
    assert all(t.shape == g2.shape for t in more) and (not more or g2.dtype == torch.bfloat16)
    dev = x.device
    dx = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    dw = torch.empty((N,), dtype=w.dtype, device=dev)
    # one CTA per partial sum, all resident at once: 3 per SM for rows of up to 4096 elements, 2 beyond
    n_partials = min(M, (3 if N <= 4096 else 2) * torch.cuda.get_device_properties(dev).multi_processor_count)
    partial = torch.empty((n_partials, N), dtype=torch.float32, device=dev)
    w = w.contiguous()
    with torch.cuda.device(dev):
        _call("coat_fp8_rmsnorm_backward", x2.data_ptr(), s2.data_ptr(), g2.data_ptr(),
              more[0].data_ptr() if len(more) > 0 else None, more[1].data_ptr() if len(more) > 1 else None,
              w.data_ptr(), v.data_ptr(), dx.data_ptr(), partial.data_ptr(), n_partials, dw.data_ptr(), M, N, QB,
              _lib.fp8_enum_of(x2), _lib.float_dtype(s2), _lib.float_dtype(g2), _lib.float_dtype(w),
              _lib.stream_ptr(dev))
    return _unflat(dx, bs), dw


def _layernorm_forward(x, s_x, w, b, QB, eps, transpose_output_2d, flags):
    (x2, s2), bs = _flat(x, s_x)
    M, N = x2.shape
    dev = x.device
    y = torch.empty((M, N), dtype=torch.float32, device=dev)   # fp32, as in the reference
    s_y = torch.empty((M,), dtype=torch.bfloat16, device=dev)
    mean = torch.empty((M,), dtype=torch.float32, device=dev)
    rstd = torch.empty((M,), dtype=torch.float32, device=dev)
    amax = _amax_word(dev)
    if w is not None:
        w, b = w.contiguous(), b.contiguous()
        assert w.dtype == b.dtype and w.numel() == N and b.numel() == N
    with torch.cuda.device(dev):
        _call("coat_fp8_layernorm_forward", x2.data_ptr(), s2.data_ptr(), None if w is None else w.data_ptr(),
              None if b is None else b.data_ptr(), y.data_ptr(), s_y.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
              amax.data_ptr(), M, N, QB, float(eps), _lib.fp8_enum_of(x2), _lib.float_dtype(s2),
              _lib.BF16 if w is None else _lib.float_dtype(w), _flags(flags), _lib.stream_ptr(dev))
        qy, s_max, qy_t = _divide(y, x2.dtype, amax, True, flags)
    if bs is not None and not transpose_output_2d:
        qy_t = qy_t.reshape(bs, -1, N)
    return _unflat(qy, bs), s_max, qy_t, mean, rstd


def fp8_layernorm_noparam_forward(x, s_x, QB, eps, transpose_output_2d=False, *, flags=None):
    qy, s_max, qy_t, mean, rstd = _layernorm_forward(x, s_x, None, None, QB, eps, transpose_output_2d, flags)
    return qy, s_max, qy_t, (mean, rstd, 8)   # 8 = num_warps of the reference, kept in the context tuple


def fp8_layernorm_param_forward(x, s_x, w, b, QB, eps, transpose_output_2d=False, *, flags=None):
    qy, s_max, qy_t, mean, rstd = _layernorm_forward(x, s_x, w, b, QB, eps, transpose_output_2d, flags)
    return qy, s_max, qy_t, (w, b, mean, rstd, 8)


def _layernorm_backward(x, s_x, g, QB, w, m, v):
    (x2, s2, g2), bs = _flat(x, s_x, g)
    M, N = g2.shape
    dev = x.device
    dx = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    dw = db = partial = None
    n_partials = 0
    if w is not None:
        w = w.contiguous()
        dw = torch.empty((N,), dtype=w.dtype, device=dev)
        db = torch.empty((N,), dtype=w.dtype, device=dev)
        n_partials = min(M, 2 * torch.cuda.get_device_properties(dev).multi_processor_count)
        partial = torch.empty((n_partials, 2, N), dtype=torch.float32, device=dev)
    P = lambda t: None if t is None else t.data_ptr()
    with torch.cuda.device(dev):
        _call("coat_fp8_layernorm_backward", x2.data_ptr(), s2.data_ptr(), g2.data_ptr(), P(w), m.data_ptr(),
              v.data_ptr(), dx.data_ptr(), P(partial), n_partials, P(dw), P(db), M, N, QB, _lib.fp8_enum_of(x2),
              _lib.float_dtype(s2), _lib.float_dtype(g2), _lib.BF16 if w is None else _lib.float_dtype(w),
              _lib.stream_ptr(dev))
    return _unflat(dx, bs), dw, db


def fp8_layernorm_noparam_backward(x, s_x, g, QB, m, v, num_warps, stochastic=False):
    if stochastic:   # the reference's branch refers to names that do not exist in its kernel and cannot run
        raise NotImplementedError("stochastic rounding of the LayerNorm input gradient is not provided")
    return _layernorm_backward(x, s_x, g, QB, None, m, v)[0]


def fp8_layernorm_param_backward(x, s_x, g, QB, w, b, m, v, num_warps):
    return _layernorm_backward(x, s_x, g, QB, w, m, v)
