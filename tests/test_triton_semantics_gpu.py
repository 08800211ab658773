"""Pins the two facts about the reference's COMPILER that decide its FP8 codes, on the actual GPU:
how Triton lowers an fp32 division (`/` and tl.fdiv) and its float -> fp8 cast.  The probe kernel
below is this repository's own four-line Triton kernel (the reference's kernels are not used); it is a
checker only, the product contains no Triton.  If the coat_b200 kernels in their default mode
reproduce the probe bit for bit, they reproduce `tl.fdiv(x, s).to(fp8)` and `(amax + 1e-10) / fp8_max`
as the reference's kernels compute them (coat/activation/real_quantization/_quantize.py:81-88)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

triton = pytest.importorskip("triton")
import triton.language as tl  # noqa: E402


@triton.jit
def _probe_kernel(x_ptr, s_ptr, y_ptr, scale_ptr, fp8_max, n, BLOCK: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    mask = offs < n
    x = tl.load(x_ptr + offs, mask=mask, other=0.0).to(tl.float32)
    s = tl.load(s_ptr).to(tl.float32)
    y = tl.fdiv(x, s).to(y_ptr.type.element_ty)
    tl.store(y_ptr + offs, y, mask=mask)
    tl.store(scale_ptr + offs, (tl.abs(x) + 1e-10) / fp8_max, mask=mask)


@pytest.mark.parametrize("fmt,dtype,fmax", [("E4M3", torch.float8_e4m3fn, 448.0), ("E5M2", torch.float8_e5m2, 57344.0)])
def test_default_mode_reproduces_triton_division_and_cast(fmt, dtype, fmax):
    import coat_b200.activation.real_quantization as r
    gen = torch.Generator().manual_seed(11)
    n = 1 << 22
    x = (torch.randn(n, generator=gen) * torch.exp(2 * torch.randn(n, generator=gen))).to(torch.bfloat16).cuda()
    for sval in (0.0123, 1.0 / 3.0, 0.00537109375, 7.3e-4):
        s = torch.tensor(sval, dtype=torch.bfloat16, device="cuda")
        y = torch.empty(n, dtype=dtype, device="cuda")
        sc = torch.empty(n, dtype=torch.float32, device="cuda")
        _probe_kernel[(triton.cdiv(n, 1024),)](x, s, y, sc, fmax, n, BLOCK=1024)
        mine, _ = r.fp8_division(x.view(-1, 4096), 16, fmt, s)
        assert torch.equal(mine.view(torch.uint8).flatten(), y.view(torch.uint8)), f"codes differ for s={sval}"
    # scales: one non-zero per 1x16 group, so the group's amax is that element
    xs = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    xs[::16] = x[::16]
    _probe_kernel[(triton.cdiv(n, 1024),)](xs, s, y, sc, fmax, n, BLOCK=1024)
    _, s_y = r.fp8_quantize(xs.view(-1, 4096), 16, fmt, torch.float32)
    assert torch.equal(s_y.flatten().view(torch.int32), sc[::16].view(torch.int32)), "group scales differ"
