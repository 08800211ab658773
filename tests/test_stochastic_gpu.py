"""GPU tests of the stochastic-rounding division (COAT_QUANT_STOCHASTIC; the reference's `stochastic=True`,
coat/activation/real_quantization/_division.py:96-150): bit-exact against the CPU oracle with IEEE division,
and the noise generator against Triton's own tl.rand on the same GPU (this repository's four-line probe
kernel; a checker only)."""
import numpy as np
import pytest
import torch

import coat_b200.activation.real_quantization as r
from coat_b200 import _lib
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def make_x(M, N, seed, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, N, generator=gen) * torch.exp(1.5 * torch.randn(M, N, generator=gen))
    x[0, :8] = 0.0
    x[1, :4] = -0.0
    return x.to(dtype)


@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_division_matches_oracle(fmt, dtype):
    x = make_x(96, 512, 31, dtype)
    s = torch.tensor(0.037, dtype=torch.bfloat16)
    want = oq.fp8_division_stochastic(x, fmt, s).view(torch.uint8)
    got, _ = r.fp8_division(x.cuda(), 16, fmt, s.cuda(), stochastic=True, flags=_lib.QUANT_IEEE_DIV)
    assert torch.equal(got.view(torch.uint8).cpu(), want)
    plain, _ = r.fp8_division(x.cuda(), 16, fmt, s.cuda(), flags=_lib.QUANT_IEEE_DIV)
    assert not torch.equal(plain.view(torch.uint8), got.view(torch.uint8))
    # zeros become the smallest subnormal with their sign (the reference's clamp from below)
    codes = got.view(torch.uint8).cpu()
    assert torch.all(codes[0, :8] == 0x01) and torch.all(codes[1, :4] == 0x81)


def test_row_stride_enters_the_noise_offset():
    big = make_x(64, 768, 32).cuda()
    view = big[:, :512]                      # row stride 768
    s = torch.tensor(0.05, dtype=torch.bfloat16)
    got, _ = r.fp8_division(view, 16, "E4M3", s.cuda(), stochastic=True, flags=_lib.QUANT_IEEE_DIV)
    want = oq.fp8_division_stochastic(view.cpu(), "E4M3", s, ld=768).view(torch.uint8)
    assert torch.equal(got.view(torch.uint8).cpu(), want)


@pytest.mark.parametrize("only_transposed", [False, True])
def test_transposed_copy_holds_the_same_codes(only_transposed):
    x = make_x(128, 256, 33).cuda()
    s = torch.tensor(0.02, dtype=torch.bfloat16, device="cuda")
    y, _ = r.fp8_division(x, 16, "E4M3", s, stochastic=True)
    out = r.fp8_division_transpose(x, 16, "E4M3", s, stochastic=True, only_transposed=only_transposed)
    y_t = out[0] if only_transposed else out[2]
    assert torch.equal(y_t.view(torch.uint8), y.view(torch.uint8).t().contiguous())
    if not only_transposed:
        assert torch.equal(out[0].view(torch.uint8), y.view(torch.uint8))


def test_pertensor_and_add_variants_pass_it_on():
    x = make_x(64, 256, 34).cuda()
    q, s_max, s_y = r.fp8_quantize_pertensor(x, 16, "E4M3", stochastic=True)
    q2, _ = r.fp8_division(x, 16, "E4M3", s_max, stochastic=True)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8))
    qa, s2, qa_t = r.fp8_quantize_pertensor_transpose(x, 16, "E4M3", stochastic=True)
    assert torch.equal(qa.view(torch.uint8), q.view(torch.uint8))
    assert torch.equal(qa_t.view(torch.uint8), q.view(torch.uint8).t().contiguous())
    b = make_x(64, 256, 35).cuda()
    y1, (qy, smax, _) = r.fp8_add_Ifp_Ifp_Ofp_Opt(x, b, 16, "E5M2", stochastic=True)
    want, _ = r.fp8_division(y1, 16, "E5M2", smax, stochastic=True)
    assert torch.equal(qy.view(torch.uint8), want.view(torch.uint8))


def test_noise_equals_triton_rand():
    triton = pytest.importorskip("triton")
    import triton.language as tl

    @triton.jit
    def _rand_probe(out_ptr, n, BLOCK: tl.constexpr):
        offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
        tl.store(out_ptr + offs, tl.rand(0, offs), mask=offs < n)

    n = 1 << 16
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    _rand_probe[(triton.cdiv(n, 1024),)](out, n, BLOCK=1024)
    assert np.array_equal(out.cpu().numpy(), oq.triton_rand(0, np.arange(n)))


def test_default_mode_equals_triton_restatement():
    """The whole operator in the default (div.full) mode against a Triton restatement of
    `tl.fdiv` + tl.rand + the perturbation + cast, on the actual GPU."""
    triton = pytest.importorskip("triton")
    import triton.language as tl

    @triton.jit
    def _probe(x_ptr, s_ptr, y_ptr, n, SUB_MIN: tl.constexpr, M_BIT: tl.constexpr, BLOCK: tl.constexpr):
        offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
        mask = offs < n
        x = tl.load(x_ptr + offs, mask=mask, other=0.0).to(tl.float32)
        q = tl.fdiv(x, tl.load(s_ptr).to(tl.float32))
        e = tl.maximum((q.to(tl.int32, bitcast=True) & 0x7F800000).to(tl.float32, bitcast=True), SUB_MIN)
        sub = e == SUB_MIN
        noise = e * tl.rand(0, offs) / tl.where(sub, 1.0, M_BIT)
        a = tl.abs(q) + noise
        a = tl.minimum(tl.maximum(a, e), tl.where(sub, M_BIT, 2.0) * e)
        a = tl.where(q.to(tl.int32, bitcast=True) < 0, -a, a)
        tl.store(y_ptr + offs, a.to(y_ptr.type.element_ty), mask=mask)

    x = make_x(256, 1024, 36).cuda()
    n = x.numel()
    for fmt, dtype, sub_min, two_m in (("E4M3", torch.float8_e4m3fn, 2.0 ** -9, 8.0), ("E5M2", torch.float8_e5m2, 2.0 ** -16, 4.0)):
        for sval in (0.0123, 1.0 / 3.0, 7.3e-4):
            s = torch.tensor(sval, dtype=torch.bfloat16, device="cuda")
            y = torch.empty(n, dtype=dtype, device="cuda")
            _probe[(triton.cdiv(n, 1024),)](x, s, y, n, SUB_MIN=sub_min, M_BIT=two_m, BLOCK=1024)
            got, _ = r.fp8_division(x, 16, fmt, s, stochastic=True)
            assert torch.equal(got.view(torch.uint8).flatten(), y.view(torch.uint8)), (fmt, sval)
