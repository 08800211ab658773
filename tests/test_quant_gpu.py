"""GPU parity tests of the quantizers, called through the python mirror of the reference API
(coat_b200.activation.real_quantization -> C ABI -> sm_100a kernels).

With COAT_QUANT_IEEE_DIV the kernels must agree with the CPU restatement (oracle/quant.py) BIT FOR BIT:
codes and stored scales.  With the default division (PTX div.full.f32, what the reference's Triton
kernels compile to, at most 2 ulp from IEEE) a code may differ from the IEEE result only where the
quotient sits within a few fp32 ulps of an FP8 rounding boundary; that set is computed and checked.
"""
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu
IEEE = 1


def ops():
    import coat_b200.activation.real_quantization as r
    from coat_b200.activation.real_quantization._quantize_transpose import fp8_quantize_transpose
    return r, fp8_quantize_transpose


def make_x(M, N, seed, dtype=torch.bfloat16, outliers=True):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, N, generator=gen)
    if outliers:
        x = torch.where(torch.rand(M, N, generator=gen) < 1e-3, x * 100, x)
    return x.to(dtype)


def u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8)


def same_bits(a, b):
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    assert a.dtype == b.dtype and a.shape == b.shape, (a.dtype, b.dtype, a.shape, b.shape)
    n = a.element_size()
    view = {1: torch.uint8, 2: torch.int16, 4: torch.int32}[n]
    bad = (a.view(view) != b.view(view)).sum().item()
    assert bad == 0, f"{bad} of {a.numel()} elements differ"


@pytest.mark.parametrize("QB", [16, 32, 64, 128])
@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("dtype,sdtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                          (torch.float16, torch.bfloat16)])
def test_group_quantize_bit_exact(QB, fmt, dtype, sdtype):
    r, _ = ops()
    x = make_x(272, 384, seed=QB, dtype=dtype)
    y, s = r.fp8_quantize(x.cuda(), QB, fmt, sdtype, flags=IEEE)
    ey, es = Q.fp8_quantize(x, QB, fmt, sdtype)
    same_bits(y, ey)
    same_bits(s, es)


def test_group_quantize_3d_and_edge_values():
    r, _ = ops()
    x = make_x(6 * 40, 64, seed=1).reshape(6, 40, 64).clone()
    x[0, 0, :16] = 0                      # all-zero group
    x[0, 1, 3] = 3e38                     # saturates to the largest finite bf16, must not overflow the cast
    x[1, 0, :16] = 1.0                    # all-equal group
    y, s = r.fp8_quantize(x.cuda(), 16, "E4M3", flags=IEEE)
    assert y.shape == (6, 40, 64) and s.shape == (6, 40, 4) and y.dtype == torch.float8_e4m3fn
    ey, es = Q.fp8_quantize(x.reshape(-1, 64), 16, "E4M3")
    same_bits(y.reshape(-1, 64), ey)
    same_bits(s.reshape(-1, 4), es)


@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("M,N", [(256, 256), (144, 80), (16, 16), (400, 4096)])
def test_pertensor_and_transpose_bit_exact(fmt, M, N):
    r, _ = ops()
    x = make_x(M, N, seed=M + N)
    q, s_max, s_y = r.fp8_quantize_pertensor(x.cuda(), 16, fmt, flags=IEEE)
    eq, es_max, es_y = Q.fp8_quantize_pertensor(x, 16, fmt)
    same_bits(s_y, es_y)
    same_bits(s_max, es_max)
    same_bits(q, eq)
    q2, s2, q_t = r.fp8_quantize_pertensor_transpose(x.cuda(), 16, fmt, flags=IEEE)
    same_bits(q2, eq)
    same_bits(s2, es_max)
    same_bits(q_t, eq.view(torch.uint8).t().contiguous().view(eq.dtype))


def test_division_variants_bit_exact():
    r, _ = ops()
    x = make_x(384, 192, seed=5)
    s = torch.tensor(0.0123, dtype=torch.bfloat16)
    e = Q.fp8_division(x, "E4M3", s)
    y, s_ret = r.fp8_division(x.cuda(), 16, "E4M3", s.cuda(), flags=IEEE)
    same_bits(y, e)
    assert s_ret.item() == s.item()
    y, _, y_t = r.fp8_division_transpose(x.cuda(), 16, "E4M3", s.cuda(), flags=IEEE)
    same_bits(y, e)
    same_bits(y_t, e.view(torch.uint8).t().contiguous().view(e.dtype))
    y_t2, _ = r.fp8_division_transpose(x.cuda(), 16, "E4M3", s.cuda(), only_transposed=True, flags=IEEE)
    same_bits(y_t2, y_t)
    # default scale: (x.abs().max() + 1e-10) / 448 evaluated in x's dtype, as torch does it
    y, s_def = r.fp8_division(x.cuda(), 16, "E4M3", flags=IEEE)
    exp_s = (x.abs().max() + 1e-10) / 448.0
    assert s_def.dtype == x.dtype and abs(s_def.float().item() - exp_s.float().item()) <= exp_s.float().item() * 2 ** -7
    same_bits(y, Q.fp8_division(x, "E4M3", s_def.cpu()))
    # 3-D input keeps its shape, the transposed copy stays 2-D
    y3, _, y3_t = r.fp8_division_transpose(x.reshape(4, 96, 192).cuda(), 16, "E4M3", s.cuda(), flags=IEEE)
    assert y3.shape == (4, 96, 192) and y3_t.shape == (192, 384)


@pytest.mark.parametrize("fmt", ["E4M3", "E5M2"])
@pytest.mark.parametrize("M,N,dtype,sdtype", [(256, 128, torch.bfloat16, torch.bfloat16),
                                              (48, 208, torch.bfloat16, torch.float32),
                                              (128, 64, torch.float32, torch.bfloat16)])
def test_quantize_transpose_bit_exact(fmt, M, N, dtype, sdtype):
    _, fp8_quantize_transpose = ops()
    x = make_x(M, N, seed=7, dtype=dtype)
    (y, s_y), (y_t, s_y_t) = fp8_quantize_transpose(x.cuda(), 16, fmt, sdtype, flags=IEEE)
    (ey, es_y), (ey_t, es_y_t) = Q.fp8_quantize_transpose(x, 16, fmt, sdtype)
    same_bits(y, ey)
    same_bits(s_y, es_y)
    same_bits(y_t, ey_t)
    same_bits(s_y_t, es_y_t)


def test_transpose_and_dequantize():
    r, _ = ops()
    gen = torch.Generator().manual_seed(9)
    codes = torch.randint(0, 256, (3, 100, 72), generator=gen, dtype=torch.uint8)
    t = r.fp8_transpose(codes.view(torch.float8_e4m3fn).cuda())
    assert t.shape == (3, 24, 300)   # the reference reshapes the (72, 300) result back to the batch
    same_bits(t.reshape(72, 300), codes.reshape(300, 72).t().contiguous().view(torch.float8_e4m3fn))
    t2 = r.fp8_transpose(codes.view(torch.float8_e4m3fn).cuda(), transpose_output_2d=True)
    assert t2.shape == (72, 300)
    x = make_x(64, 256, seed=2)
    q, s = Q.fp8_quantize(x, 32, "E5M2")
    d = r.fp8_dequantize(q.cuda(), s.cuda(), 32)
    same_bits(d, Q.fp8_dequantize(q, s, 32))


def test_default_division_differs_only_at_rounding_boundaries():
    """div.full.f32 (default, the reference's division) vs IEEE division: stored bf16 scales identical,
    codes different only where x/s is within 6 fp32 ulps of a rounding boundary.  With bf16 inputs many
    quotients are EXACT ties (e.g. 19.0 between the codes for 18 and 20), which IEEE division resolves to
    even and an approximate division to either side, so the rate is not negligible: below 2e-3 here."""
    r, fp8_quantize_transpose = ops()
    x = make_x(2048, 4096, seed=1)
    y, s = r.fp8_quantize(x.cuda(), 16, "E4M3")
    ey, es = Q.fp8_quantize(x, 16, "E4M3")
    same_bits(s, es)
    diff = u8(y) != u8(ey)
    quot = (x.float().reshape(2048, 256, 16) / Q.group_scales(x, 16, "E4M3").unsqueeze(-1)).reshape(2048, 4096)
    near = Q.near_rounding_boundary(quot, "E4M3", ulps=6)
    assert not (diff & ~near).any()
    assert diff.float().mean().item() < 2e-3
    q, s_max, _ = r.fp8_quantize_pertensor(x.cuda(), 16, "E4M3")
    eq, es_max, _ = Q.fp8_quantize_pertensor(x, 16, "E4M3")
    same_bits(s_max, es_max)
    diff = u8(q) != u8(eq)
    near = Q.near_rounding_boundary(x.float() / es_max.float(), "E4M3", ulps=6)
    assert not (diff & ~near).any() and diff.float().mean().item() < 2e-3


def test_full_size_properties():
    """The benchmark configuration (8192 tokens x 4096, 0.1 % outliers x100): properties that need no
    CPU pass over 33.5 M elements twice: transposed codes are the transpose of the straight codes, the
    per-tensor scale is the maximum group scale, and dequantisation error stays within half a step."""
    r, fp8_quantize_transpose = ops()
    x = make_x(8192, 4096, seed=1).cuda()
    q, s_max, q_t = r.fp8_quantize_pertensor_transpose(x, 16, "E4M3")
    assert torch.equal(q.view(torch.uint8).t(), q_t.view(torch.uint8))
    q2, s_max2, s_y = r.fp8_quantize_pertensor(x, 16, "E4M3")
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8)) and s_max == s_max2 == s_y.max()
    err = (q.float() * s_max.float() - x.float()).abs()
    assert (err <= 0.0625 * x.float().abs() + s_max.float() * 2 ** -9 + 1e-6).all()   # 3 mantissa bits / subnormal step
    (y, s_y), (y_t, s_y_t) = fp8_quantize_transpose(x, 16, "E4M3")
    yg, sg = r.fp8_quantize(x, 16, "E4M3")
    assert torch.equal(y.view(torch.uint8), yg.view(torch.uint8)) and torch.equal(s_y, sg)
    ytg, stg = r.fp8_quantize(x.t().contiguous(), 16, "E4M3")
    assert torch.equal(y_t.view(torch.uint8), ytg.view(torch.uint8)) and torch.equal(s_y_t, stg)
    d = r.fp8_dequantize(y, s_y, 16)
    assert ((d.float() - x.float()).abs() <= 0.07 * x.float().abs() + s_y.float().repeat_interleave(16, 1) * 2 ** -9).all()


def test_quantizer_error_conventions():
    r, fp8_quantize_transpose = ops()
    x = make_x(32, 48, seed=0).cuda()
    with pytest.raises(RuntimeError):           # N not a multiple of QB
        r.fp8_quantize(x, 32, "E4M3")
    with pytest.raises(RuntimeError):           # the fused transpose quantizer fixes 1x16 groups
        fp8_quantize_transpose(x, 32, "E4M3")
    with pytest.raises(RuntimeError, match="CUDA"):
        r.fp8_quantize(x.cpu(), 16, "E4M3")
    y, s = r.fp8_quantize(x[:0], 16, torch.float8_e5m2)   # empty input, dtype given as torch dtype
    assert y.shape == (0, 48) and y.dtype == torch.float8_e5m2


# ---- 128-wide granularities (block-scaled linear layer) --------------------------------------------
@pytest.mark.parametrize("fp8type", [torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("shape", [(128, 128), (256, 384), (1024, 512)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_block128_quantizers_bit_exact_ieee(fp8type, shape, dtype):
    from coat_b200 import _lib
    from coat_b200.activation.real_quantization import (fp8_quantize_perblock, fp8_quantize_perblock_transpose,
                                                        fp8_quantize_perblock_transpose_pergroup,
                                                        fp8_quantize_transpose)
    from oracle import quant as OQ
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(shape, generator=gen)
    x = torch.where(torch.rand(shape, generator=gen) < 1e-3, x * 100, x).to(dtype)
    want = OQ.fp8_quantize_block128(x, fp8type, torch.float32)
    xd = x.cuda()
    F = _lib.QUANT_IEEE_DIV

    def same(got, key):
        q, s = got
        wq, ws = want[key]
        assert torch.equal(q.cpu().view(torch.uint8), wq.view(torch.uint8)), key
        assert torch.equal(s.cpu(), ws), key

    same(fp8_quantize_perblock(xd, 128, fp8type, scale_dtype=torch.float32, flags=F), "block")
    b, bt = fp8_quantize_perblock_transpose(xd, 128, fp8type, scale_dtype=torch.float32, flags=F)
    same(b, "block"); same(bt, "block_t")
    same(fp8_quantize_perblock_transpose(xd, 128, fp8type, scale_dtype=torch.float32, only_transposed=True, flags=F), "block_t")
    b, bt, pg = fp8_quantize_perblock_transpose_pergroup(xd, 128, fp8type, scale_dtype=torch.float32, flags=F)
    same(b, "block"); same(bt, "block_t"); same(pg, "rows")
    r, ct = fp8_quantize_transpose(xd, 128, fp8type, scale_dtype=torch.float32, flags=F)
    same(r, "rows"); same(ct, "cols_t")


def test_block128_default_division_differs_only_at_rounding_boundaries():
    from coat_b200.activation.real_quantization import fp8_quantize_perblock
    from oracle import quant as OQ
    gen = torch.Generator().manual_seed(12)
    x = torch.randn(512, 512, generator=gen).to(torch.bfloat16)
    q, s = fp8_quantize_perblock(x.cuda(), 128, "E4M3", scale_dtype=torch.float32)
    wq, ws = OQ.fp8_quantize_block128(x, torch.float8_e4m3fn)["block"]
    assert torch.allclose(s.cpu(), ws, rtol=2e-7)
    diff = q.cpu().view(torch.uint8) != wq.view(torch.uint8)
    assert diff.float().mean() < 2e-3
    assert (q.cpu().float() - wq.float()).abs().max() <= 32   # one code step at most


def test_block128_rejects_ragged_shapes():
    from coat_b200.activation.real_quantization import fp8_quantize_perblock
    with pytest.raises(RuntimeError):
        fp8_quantize_perblock(torch.zeros(128, 192, dtype=torch.bfloat16, device="cuda"), 128, "E4M3")
    with pytest.raises(RuntimeError):
        fp8_quantize_perblock(torch.zeros(128, 128, dtype=torch.bfloat16, device="cuda"), 64, "E4M3")


@pytest.mark.parametrize("QB", [16, 32, 128])
@pytest.mark.parametrize("dtype,scale_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                               (torch.float16, torch.bfloat16)])
def test_one_launch_pertensor_bit_exact(QB, dtype, scale_dtype):
    """The cooperative one-launch per-tensor quantize (amax, grid barrier, division re-reading x backwards):
    group sizes, input and scale dtypes, a row count that leaves the last CTA a ragged slice, a row stride."""
    r, _ = ops()
    from coat_b200 import _lib
    M, N = 1000, 384
    big = make_x(M, N + 128, seed=QB, dtype=dtype)
    for x in (big[:, :N].contiguous(), big[:, :N]):          # contiguous, and with a row stride of N + 128
        q, s_max, s_y = r.fp8_quantize_pertensor(x.cuda() if x.is_contiguous() else big.cuda()[:, :N], QB, "E4M3",
                                                 scale_dtype=scale_dtype, flags=IEEE)
        eq, es_max, es_y = Q.fp8_quantize_pertensor(x.contiguous(), QB, "E4M3", scale_dtype=scale_dtype)
        same_bits(s_y, es_y)
        same_bits(s_max, es_max)
        same_bits(q, eq)
    assert _lib.lib().coat_fp8_quantize_device_status() == 0


def test_one_launch_pertensor_many_trips_equals_two_pass():
    """A matrix large enough that every CTA walks its slice in several trips (persistent grid): the result
    equals the two-launch path (group scales + amax, then division), 3-D input included."""
    r, _ = ops()
    x = make_x(4 * 4096, 2048, seed=77).cuda().view(4, 4096, 2048)
    q, s_max, s_y = r.fp8_quantize_pertensor(x, 16, "E5M2")
    q2, s_max2, q_t = r.fp8_quantize_pertensor_transpose(x, 16, "E5M2", transpose_output_2d=True)
    assert q.shape == (4, 4096, 2048) and s_y.shape == (4, 4096, 128)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8)) and s_max == s_max2
    assert torch.equal(q_t.view(torch.uint8), q.view(torch.uint8).view(-1, 2048).t())
    _, s_ref = r.fp8_quantize(x, 16, "E5M2")
    assert torch.equal(s_y, s_ref) and s_max == s_y.max()
    # both one-launch kernels against the plain division kernel with the same scale
    q3, _ = r.fp8_division(x, 16, "E5M2", s_max)
    assert torch.equal(q.view(torch.uint8), q3.view(torch.uint8))
    from coat_b200 import _lib
    assert _lib.lib().coat_fp8_quantize_device_status() == 0


@pytest.mark.parametrize("transposed", [False, True])
def test_one_launch_pertensor_timeout_is_reported_and_heals(transposed):
    """The grid barrier of the one-launch kernels is bounded.  With the bound lowered to zero polls (a diagnostic
    switch; nothing waits, nothing hangs) the first CTAs to arrive give up: the status word must read
    COAT_E_TIMEOUT, the sync words must be back at zero, and the next call with the normal bound on the SAME sync
    words must give the right result."""
    r, _ = ops()
    from coat_b200 import _lib
    from coat_b200.activation.real_quantization import _ops
    L = _lib.lib()
    x = make_x(2048, 1024, seed=5).cuda()
    fn = (lambda: r.fp8_quantize_pertensor_transpose(x, 16, "E4M3")) if transposed else \
         (lambda: r.fp8_quantize_pertensor(x, 16, "E4M3"))
    good = fn()
    assert L.coat_fp8_quantize_device_status() == 0
    words = _ops._sync_words(x.device)[1]
    assert L.coat_fp8_quantize_set_barrier_limit(0) == 0
    try:
        fn()
        assert L.coat_fp8_quantize_device_status() == _lib.E_TIMEOUT
    finally:
        assert L.coat_fp8_quantize_set_barrier_limit(-1) == 0
    assert words.tolist()[:3] == [0, 0, 0], "a call that timed out must leave the sync words clean"
    again = fn()
    assert L.coat_fp8_quantize_device_status() == 0
    for a, b in zip(good, again):
        assert torch.equal(a.view(torch.uint8) if a.dtype.itemsize == 1 else a, b.view(torch.uint8) if b.dtype.itemsize == 1 else b)


def test_one_launch_transposed_falls_back_for_ragged_row_counts():
    """M not a multiple of 16: the operator takes the two-call path; results agree with the straight one-launch kernel."""
    r, _ = ops()
    x = make_x(1004, 256, seed=78).cuda()
    q, s_max, q_t = r.fp8_quantize_pertensor_transpose(x, 16, "E4M3")
    q2, s_max2, _ = r.fp8_quantize_pertensor(x, 16, "E4M3")
    assert s_max == s_max2 and torch.equal(q.view(torch.uint8), q2.view(torch.uint8))
    assert torch.equal(q_t.view(torch.uint8), q.view(torch.uint8).t())


def test_one_launch_pertensor_replays_from_a_cuda_graph():
    """Cooperative launches inside a captured graph: replays (with the input changed in place between them) equal
    the eager results, so the sync words really are zero again after every launch."""
    r, _ = ops()
    x = make_x(2048, 1024, seed=90).cuda()
    x2 = make_x(2048, 1024, seed=91).cuda()
    buf = x.clone()
    r.fp8_quantize_pertensor(buf, 16, "E4M3")               # first use outside the capture
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        q, s_max, s_y = r.fp8_quantize_pertensor(buf, 16, "E4M3")
        qa, sa, qa_t = r.fp8_quantize_pertensor_transpose(buf, 16, "E4M3")
    for src in (x, x2, x):
        buf.copy_(src)
        g.replay()
        torch.cuda.synchronize()
        eq, es_max, es_y = r.fp8_quantize_pertensor(src, 16, "E4M3")
        assert torch.equal(q.view(torch.uint8), eq.view(torch.uint8)) and s_max == es_max and torch.equal(s_y, es_y)
        assert torch.equal(qa.view(torch.uint8), eq.view(torch.uint8)) and sa == es_max
        assert torch.equal(qa_t.view(torch.uint8), eq.view(torch.uint8).t())
