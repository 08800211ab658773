"""The allocation-free per-tensor quantize (coat_fp8_quantize_pertensor_static) against the ordinary
two-call path.

Some hosts cannot allocate on the device where they quantize (a fixed memory budget, no caching
allocator, a section where cudaMalloc would stall the GPU), so that entry point keeps its scratch in
a static device array inside the library.  The array is shared by all calls and keeps the previous
call's contents, which is exactly what could go wrong: the test therefore makes two calls in a row on
different data (the second smaller, so stale partial maxima of the first sit beyond the slots it uses)
and requires both to match the ordinary path bit for bit.  It calls through the C ABI with raw
pointers; the output buffers are made by the test, the entry point itself receives no scratch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _static_quantize(x, fmt_name, want_t=True):
    from coat_b200 import _lib
    M, N = x.shape
    fmt, dt = _lib.fp8_format(fmt_name)
    y = torch.empty((M, N), dtype=dt, device=x.device)
    y_t = torch.empty((N, M), dtype=dt, device=x.device) if want_t else None
    s = torch.empty((), dtype=torch.bfloat16, device=x.device)
    rc = _lib.lib().coat_fp8_quantize_pertensor_static(
        x.data_ptr(), y.data_ptr(), None if y_t is None else y_t.data_ptr(), s.data_ptr(), M, N, x.stride(0),
        fmt, _lib.float_dtype(x), _lib.BF16, 0, _lib.stream_ptr(x.device))
    return rc, y, s, y_t


def test_static_scratch_variant_matches_ordinary_path_twice_in_a_row():
    import coat_b200.activation.real_quantization as r
    gen = torch.Generator().manual_seed(21)
    big = (torch.randn(2048, 1024, generator=gen) * 7.0).to(torch.bfloat16).cuda()      # 128 partial slots
    small = (torch.randn(64, 256, generator=gen) * 0.01).to(torch.bfloat16).cuda()      # 1 partial slot, tiny amax
    for x in (big, small):
        rc, y, s, y_t = _static_quantize(x, "E4M3")
        assert rc == 0
        ey, es, ey_t = r.fp8_quantize_pertensor_transpose(x, 16, "E4M3")
        torch.cuda.synchronize()
        assert torch.equal(s.view(torch.int16), es.view(torch.int16))
        assert torch.equal(y.view(torch.uint8), ey.view(torch.uint8))
        assert torch.equal(y_t.view(torch.uint8), ey_t.view(torch.uint8))
    # straight codes only, E5M2
    rc, y, s, _ = _static_quantize(big, "E5M2", want_t=False)
    ey, es, _ = r.fp8_quantize_pertensor(big, 16, "E5M2")
    assert rc == 0 and torch.equal(y.view(torch.uint8), ey.view(torch.uint8)) and s == es


def test_static_scratch_variant_rejects_oversized_input():
    from coat_b200 import _lib
    # 8192 x 8208 = 67 239 936 elements, just above the 67 108 864 the static array can serve; the call
    # must refuse before touching memory, so the buffers only need to exist, not to be that large
    x = torch.empty(16, 8208, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(16, dtype=torch.uint8, device="cuda")
    s = torch.empty((), dtype=torch.bfloat16, device="cuda")
    rc = _lib.lib().coat_fp8_quantize_pertensor_static(x.data_ptr(), y.data_ptr(), None, s.data_ptr(), 8192, 8208,
                                                       8208, _lib.E4M3, _lib.BF16, _lib.BF16, 0,
                                                       _lib.stream_ptr(x.device))
    assert rc == -7   # COAT_E_TOOBIG
    with pytest.raises(RuntimeError, match="maximum"):
        _lib.check(rc, "quantize_pertensor_static")


def test_static_scratch_variant_rejects_stochastic_rounding():
    """Round-to-nearest only: the stochastic flag is refused (COAT_E_BADARG), not silently dropped."""
    from coat_b200 import _lib
    x = torch.zeros(16, 64, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(16, 64, dtype=torch.uint8, device="cuda")
    s = torch.empty((), dtype=torch.bfloat16, device="cuda")
    rc = _lib.lib().coat_fp8_quantize_pertensor_static(x.data_ptr(), y.data_ptr(), None, s.data_ptr(), 16, 64, 64,
                                                       _lib.E4M3, _lib.BF16, _lib.BF16, _lib.QUANT_STOCHASTIC,
                                                       _lib.stream_ptr(x.device))
    assert rc == _lib.E_BADARG
