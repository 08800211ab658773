"""GPU parity tests of the fused FP8 AdamW kernels, called through the C ABI
(coat_b200.optimizer.qoptim_cuda -> libcoat_b200.so).

Checkers, strongest first:
  1. the reference's own CUDA extension compiled for sm_100a by oracle/build_ref.py (bit level),
  2. the C restatement oracle/fp8_adamw_oracle.c (bit level where no libm/libdevice call is
     involved, stated tolerances elsewhere),
  3. the golden vectors made from the reference's pure-PyTorch expectation.
"""
import os

import numpy as np
import pytest
import torch

from _ref import load_ref_qoptim
from oracle import adamw as O

pytestmark = pytest.mark.gpu

HYPER = dict(beta1=0.9, beta2=0.95, lr=1e-4, wd=0.1, eps=1e-8)
KEYS = ("p", "m", "v", "s_m", "k_m", "r_m", "s_v", "k_v", "r_v")
STATE_KEYS = KEYS[1:]          # everything that is quantised or derived from group statistics
EXACT_POW = 1                  # COAT_ADAMW_EXACT_POW


def assert_weights_close(a, b, lr, what=""):
    """Tolerance of the fp32 weights on the guarded fast path (stated up front): the approximate
    moments carry a relative error of a few 1e-6, so one update differs by at most 1e-5 of its size
    (taken as lr * 10), plus two ulps of the weight itself.  Codes, scales, exponents and
    sqrt(max*min) are NOT covered by any tolerance: they must be bit-identical."""
    x, y = a["p"].float().cpu(), b["p"].float().cpu()
    bad = (x - y).abs() > 2.4e-7 * y.abs() + 1e-5 * lr * 10
    bad &= ~(x.isnan() & y.isnan())
    assert not bad.any(), f"{what}: weights differ beyond tolerance in {int(bad.sum())} places"


def mine():
    from coat_b200.optimizer import qoptim_cuda
    return qoptim_cuda


def fresh(n, seed=0, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    G = (n + 127) // 128
    st = dict(p=(torch.randn(n, generator=gen) * 0.02).to(dtype), m=torch.zeros(n, dtype=torch.uint8),
              v=torch.zeros(n, dtype=torch.uint8), s_m=torch.zeros(G), k_m=torch.ones(G), r_m=torch.ones(G),
              s_v=torch.zeros(G), k_v=torch.ones(G), r_v=torch.ones(G))
    return st, gen


def to(st, device):
    return {k: v.clone().to(device) for k, v in st.items()}


def expand_step(mod, st, g, step, hyper=HYPER, fp8_views=False, **kw):
    m = st["m"].view(torch.float8_e4m3fn) if fp8_views else st["m"]
    v = st["v"].view(torch.float8_e4m3fn) if fp8_views else st["v"]
    mod.fp8_adamw_expand_step(st["p"], g, m, st["s_m"], st["k_m"], st["r_m"], v, st["s_v"], st["k_v"], st["r_v"],
                              hyper["beta1"], hyper["beta2"], hyper["lr"], hyper["wd"], hyper["eps"], step, 128,
                              16, **kw)


def plain_step(mod, st, g, step, hyper=HYPER, fp8_views=False, **kw):
    m = st["m"].view(torch.float8_e4m3fn) if fp8_views else st["m"]
    v = st["v"].view(torch.float8_e4m3fn) if fp8_views else st["v"]
    mod.fp8_adamw_step(st["p"], g, m, st["s_m"], v, st["s_v"], hyper["beta1"], hyper["beta2"], hyper["lr"],
                       hyper["wd"], hyper["eps"], step, 128, **kw)


def bits(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float32:
        return t.view(torch.int32)
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16)
    return t.view(torch.uint8)


def assert_bit_equal(a, b, keys=KEYS, what=""):
    for k in keys:
        x, y = bits(a[k]), bits(b[k])
        # NaN payloads aside, every bit must agree
        bad = (x != y)
        if a[k].dtype.is_floating_point:
            bad &= ~(a[k].cpu().isnan() & b[k].cpu().isnan())
        assert not bad.any(), f"{what}: {k} differs in {int(bad.sum())} of {bad.numel()} places"


# ---------------------------------------------------------------------------------------------
# 1. bit-exact against the reference's own kernel
# ---------------------------------------------------------------------------------------------

@pytest.mark.parametrize("n", [1, 127, 128, 129, 128 * 7 + 5, 4096 * 64])
def test_expand_bit_exact_vs_reference_kernel(n):
    ref = load_ref_qoptim()
    if ref is None:
        pytest.skip("oracle/_ref/qoptim_cuda.so not built (python oracle/build_ref.py)")
    st0, gen = fresh(n, seed=n % 7)
    a, b, x = to(st0, "cuda"), to(st0, "cuda"), to(st0, "cuda")
    for step in range(1, 11):
        g = (torch.randn(n, generator=gen) * 1e-3).cuda()
        expand_step(mine(), a, g, step)                      # guarded fast path (default)
        expand_step(mine(), x, g, step, flags=EXACT_POW)     # exact pow everywhere
        expand_step(ref, b, g, step, fp8_views=True)
        torch.cuda.synchronize()
        assert_bit_equal(x, b, what=f"exact n={n} step={step}")
        assert_bit_equal(a, b, keys=STATE_KEYS, what=f"fast n={n} step={step}")
        assert_weights_close(a, b, HYPER["lr"], what=f"fast n={n} step={step}")
        a["p"].copy_(b["p"])   # keep the three runs on the same trajectory


@pytest.mark.parametrize("n", [129, 4096 * 16 + 3, 4096 * 512])
def test_plain_bit_exact_vs_reference_kernel(n):
    """The step without expansion.  Exact mode: every array bit-identical to the reference's kernel.  Default mode
    (approximate square root / reciprocal in the weight update, guarded reciprocal in the requantisation): codes
    and scales bit-identical, weights within the tolerance stated for the default mode."""
    ref = load_ref_qoptim()
    if ref is None:
        pytest.skip("oracle/_ref/qoptim_cuda.so not built (python oracle/build_ref.py)")
    st0, gen = fresh(n, seed=11)
    a, b, x = to(st0, "cuda"), to(st0, "cuda"), to(st0, "cuda")
    for step in range(1, 11):
        g = (torch.randn(n, generator=gen) * 1e-3).cuda()
        if step == 4:   # a few adversarial groups: all zero, all equal, huge dynamic range
            gv = g[: (n // 128) * 128].view(-1, 128)
            gv[0] = 0.0
            if gv.shape[0] > 2:
                gv[1] = 3e-4
                gv[2] *= torch.logspace(-12, 2, 128, device="cuda")
        plain_step(mine(), a, g, step)
        plain_step(mine(), x, g, step, flags=EXACT_POW)
        plain_step(ref, b, g, step, fp8_views=True)
        torch.cuda.synchronize()
        assert_bit_equal(x, b, keys=("p", "m", "v", "s_m", "s_v"), what=f"plain exact n={n} step={step}")
        assert_bit_equal(a, b, keys=("m", "v", "s_m", "s_v"), what=f"plain default n={n} step={step}")
        assert_weights_close(a, b, HYPER["lr"], what=f"plain default n={n} step={step}")
        a["p"].copy_(b["p"])


def test_expand_benchmark_tensor_bit_exact_vs_reference_kernel():
    """The optimizer benchmark case at its full size: one fp32 parameter of 4096 x 4096, gradients N(0, 1e-3) drawn
    step by step from seed 0, lr 1e-4, betas (0.9, 0.95), weight decay 0.1, 10 steps from a fresh state; all nine
    arrays compared with the reference's compiled kernel after every step (exact mode: every bit; default mode:
    every bit of the eight state arrays, weights within the stated tolerance)."""
    ref = load_ref_qoptim()
    if ref is None:
        pytest.skip("oracle/_ref/qoptim_cuda.so not built (python oracle/build_ref.py)")
    n = 4096 * 4096
    gen = torch.Generator().manual_seed(0)
    G = n // 128
    st0 = dict(p=torch.randn(4096, 4096, generator=gen).mul_(0.02).view(-1), m=torch.zeros(n, dtype=torch.uint8),
               v=torch.zeros(n, dtype=torch.uint8), s_m=torch.zeros(G), k_m=torch.ones(G), r_m=torch.ones(G),
               s_v=torch.zeros(G), k_v=torch.ones(G), r_v=torch.ones(G))
    a, b, x = to(st0, "cuda"), to(st0, "cuda"), to(st0, "cuda")
    for step in range(1, 11):
        g = torch.randn(4096, 4096, generator=gen).mul_(1e-3).view(-1).cuda()
        expand_step(mine(), a, g, step)
        expand_step(mine(), x, g, step, flags=EXACT_POW)
        expand_step(ref, b, g, step, fp8_views=True)
        torch.cuda.synchronize()
        for k in KEYS:   # compared on the device: 16.7 M elements per array
            same = torch.equal(x[k].view(torch.uint8), b[k].view(torch.uint8))
            assert same, f"exact mode, step {step}: {k} differs from the reference kernel"
        for k in STATE_KEYS:
            same = torch.equal(a[k].view(torch.uint8), b[k].view(torch.uint8))
            assert same, f"default mode, step {step}: {k} differs from the reference kernel"
        bad = (a["p"] - b["p"]).abs() > 2.4e-7 * b["p"].abs() + 1e-5 * HYPER["lr"] * 10
        assert not bool(bad.any()), f"default mode, step {step}: weights outside tolerance"
        a["p"].copy_(b["p"])


def adversarial_grads(n, gen, step):
    """Gradients that exercise the order-dependent minimum (exact zeros at chosen lanes), all-zero
    groups, all-equal groups and large dynamic range."""
    g = torch.randn(n, generator=gen) * 1e-3
    G = n // 128
    gv = g[: G * 128].view(G, 128)
    for grp in range(G):
        kind = grp % 8
        if kind == 1:
            gv[grp, [0]] = 0.0
        elif kind == 2:
            gv[grp, [5, 8, 16, 24, 32, 64, 96]] = 0.0
        elif kind == 3:
            gv[grp] = 0.0  # e.g. the embedding row of a token that never occurs
        elif kind == 4:
            gv[grp] = 3e-4  # all equal: ratio 1, exponent +inf
        elif kind == 5:
            gv[grp] *= torch.logspace(-12, 2, 128)
        elif kind == 6 and step % 2 == 0:
            gv[grp] = 0.0
    return g


def test_expand_adversarial_bit_exact_vs_reference_kernel():
    ref = load_ref_qoptim()
    if ref is None:
        pytest.skip("oracle/_ref/qoptim_cuda.so not built (python oracle/build_ref.py)")
    n = 128 * 64 + 77
    st0, gen = fresh(n, seed=5)
    a, b, x = to(st0, "cuda"), to(st0, "cuda"), to(st0, "cuda")
    for step in range(1, 9):
        g = adversarial_grads(n, gen, step).cuda()
        expand_step(mine(), a, g, step)
        expand_step(mine(), x, g, step, flags=EXACT_POW)
        expand_step(ref, b, g, step, fp8_views=True)
        torch.cuda.synchronize()
        assert_bit_equal(x, b, what=f"adversarial exact step={step}")
        assert_bit_equal(a, b, keys=STATE_KEYS, what=f"adversarial fast step={step}")
        assert_weights_close(a, b, HYPER["lr"], what=f"adversarial fast step={step}")
        a["p"].copy_(b["p"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_expand_half_precision_params_bit_exact_vs_reference_kernel(dtype):
    ref = load_ref_qoptim()
    if ref is None:
        pytest.skip("oracle/_ref/qoptim_cuda.so not built (python oracle/build_ref.py)")
    n = 128 * 33 + 2
    st0, gen = fresh(n, seed=2, dtype=dtype)
    a, b = to(st0, "cuda"), to(st0, "cuda")
    for step in range(1, 6):
        g = (torch.randn(n, generator=gen) * 1e-3).to(dtype).cuda()
        expand_step(mine(), a, g, step)
        expand_step(ref, b, g, step, fp8_views=True)
        torch.cuda.synchronize()
        assert_bit_equal(a, b, what=f"{dtype} step={step}")


def _soak_grads(kind, n, gen):
    g = torch.randn(n, generator=gen)
    if kind == "gauss_1e-3":
        return g * 1e-3
    if kind == "gauss_1e-8":
        return g * 1e-8
    if kind == "gauss_1e2":
        return g * 1e2
    if kind == "heavy_tail":
        return g * torch.exp(3 * torch.randn(n, generator=gen)) * 1e-4
    if kind == "sparse":
        return g * 1e-3 * (torch.rand(n, generator=gen) < 0.3)
    if kind == "row_scaled":
        return (g.view(-1, 128) * torch.logspace(-9, 1, n // 128).view(-1, 1)).reshape(n)
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["gauss_1e-3", "gauss_1e-8", "gauss_1e2", "heavy_tail", "sparse", "row_scaled"])
def test_guarded_fast_path_long_soak(kind):
    """Volume test of the guarded fast path: 16.7 M parameters x 64 steps = 1.07e9 element-steps per distribution
    (6.4e9 in all), gradients drawn on the device, default mode against the exact mode of the same library (which
    the tests above tie to the reference's kernel bit for bit).  Every code, scale, exponent and sqrt(max*min)
    must be identical after every step; compared on the device."""
    n = 4096 * 4096
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(1234)
    G = n // 128

    def draw():
        g = torch.randn(n, generator=gen, device=dev)
        if kind == "gauss_1e-3":
            return g * 1e-3
        if kind == "gauss_1e-8":
            return g * 1e-8
        if kind == "gauss_1e2":
            return g * 1e2
        if kind == "heavy_tail":
            return g * torch.exp(3 * torch.randn(n, generator=gen, device=dev)) * 1e-4
        if kind == "sparse":
            return g * 1e-3 * (torch.rand(n, generator=gen, device=dev) < 0.3)
        return (g.view(-1, 128) * torch.logspace(-9, 1, G, device=dev).view(-1, 1)).reshape(n)

    st = dict(p=torch.randn(n, generator=gen, device=dev) * 0.02, m=torch.zeros(n, dtype=torch.uint8, device=dev),
              v=torch.zeros(n, dtype=torch.uint8, device=dev), s_m=torch.zeros(G, device=dev),
              k_m=torch.ones(G, device=dev), r_m=torch.ones(G, device=dev), s_v=torch.zeros(G, device=dev),
              k_v=torch.ones(G, device=dev), r_v=torch.ones(G, device=dev))
    a, x = {k: v.clone() for k, v in st.items()}, {k: v.clone() for k, v in st.items()}
    for step in range(1, 65):
        g = draw()
        expand_step(mine(), a, g, step)
        expand_step(mine(), x, g, step, flags=EXACT_POW)
        for k in STATE_KEYS:
            if a[k].dtype == torch.uint8:
                diff = a[k] != x[k]
            else:   # NaN payloads aside, every bit must agree
                diff = (a[k].view(torch.int32) != x[k].view(torch.int32)) & ~(a[k].isnan() & x[k].isnan())
            assert not bool(diff.any()), f"{kind} step {step}: {k} differs in {int(diff.sum())} places"
        bad = (a["p"] - x["p"]).abs() > 2.4e-7 * x["p"].abs() + 1e-5 * HYPER["lr"] * 10
        bad &= ~(a["p"].isnan() & x["p"].isnan())
        assert not bool(bad.any()), f"{kind} step {step}: weights outside tolerance"
        a["p"].copy_(x["p"])
    from coat_b200 import _lib
    assert _lib.lib().coat_fp8_adamw_device_status() == 0


@pytest.mark.parametrize("kind", ["gauss_1e-3", "gauss_1e-8", "gauss_1e2", "heavy_tail", "sparse", "row_scaled"])
def test_guarded_fast_path_equals_exact_path(kind):
    """Soak test of the guarded fast path against the exact path of the same library, over value
    distributions a training run can produce (tiny / huge gradients, heavy tails, exact zeros, rows
    of very different scale): every code, scale, exponent and sqrt(max*min) bit-identical at every
    step, weights inside the stated tolerance; and the fast path must actually be taken."""
    import ctypes
    from coat_b200 import _lib
    n = 128 * 8192
    st0, gen = fresh(n, seed=17)
    a, x = to(st0, "cuda"), to(st0, "cuda")
    counters = torch.zeros(8, dtype=torch.int64, device="cuda")
    lr = HYPER["lr"]
    try:
        for step in range(1, 9):
            g = _soak_grads(kind, n, gen).cuda()
            _lib.lib().coat_fp8_adamw_debug_counters(ctypes.c_void_p(counters.data_ptr()))
            expand_step(mine(), a, g, step)
            torch.cuda.synchronize()
            _lib.lib().coat_fp8_adamw_debug_counters(None)
            expand_step(mine(), x, g, step, flags=EXACT_POW)
            torch.cuda.synchronize()
            assert_bit_equal(a, x, keys=STATE_KEYS, what=f"{kind} step={step}")
            assert_weights_close(a, x, lr, what=f"{kind} step={step}")
            a["p"].copy_(x["p"])
    finally:
        _lib.lib().coat_fp8_adamw_debug_counters(None)
    fast, exact = counters[0].item(), counters[1].item()
    assert fast + exact == 8 * (n // 128)
    # Step 1 starts from an all-zero state (exact path).  Groups that hold exact zeros take the exact path
    # by design; so do groups whose smallest |m'| is below the group-wide error bound (about 5e-6 of the
    # largest), which heavy-tailed gradients produce in roughly half of the groups.
    floor = {"sparse": 0.0, "heavy_tail": 0.3}.get(kind, 0.8)
    assert fast >= floor * 7 * (n // 128), (fast, exact)
    used = counters[6:8].to(torch.int32).view(torch.float32)
    assert (used < 1.0).all(), f"approximation error exceeded its modelled bound: {used.tolist()}"
    assert _lib.lib().coat_fp8_adamw_device_status() == 0


# ---------------------------------------------------------------------------------------------
# 2. against the C restatement
# ---------------------------------------------------------------------------------------------

def test_plain_vs_c_oracle_states_bit_exact():
    """No libm/libdevice call touches the moments of the plain kernel, so codes and scales must be
    bit-identical to the C restatement; the weights pass through powf(beta, step) (host libm there,
    libdevice here): tolerance 1e-6 relative to |weight| + lr (the size of one update)."""
    n = 128 * 50 + 9
    st0, gen = fresh(n, seed=3)
    a, c = to(st0, "cuda"), to(st0, "cpu")
    for step in range(1, 11):
        g = torch.randn(n, generator=gen) * 1e-3
        plain_step(mine(), a, g.cuda(), step)
        plain_step(O, c, g, step)
        torch.cuda.synchronize()
        assert_bit_equal(a, c, keys=("m", "v", "s_m", "s_v"), what=f"plain step={step}")
        assert ((a["p"].cpu() - c["p"]).abs() <= 1e-6 * (c["p"].abs() + HYPER["lr"])).all()


def test_expand_vs_c_oracle_tolerance():
    """Expansion kernel vs C restatement: host powf/log2f differ from libdevice in the last place, so
    (tolerances fixed here) exponents equal on >= 99.9 % of groups, scales and sqrt-min-max rtol 1e-4
    on >= 99 % (1e-2 on all) of the groups with equal exponent, >= 99.5 % identical codes there and never more than one code
    step apart; weights: >= 99.5 % within 1e-5 relative (+1e-8), and every weight within 0.2 * lr (where
    a code differs by one step the dequantised moment moves by up to 1/8, and with it that element's
    update, whose size is about lr)."""
    n = 4096 * 64
    st0, gen = fresh(n, seed=4)
    a, c = to(st0, "cuda"), to(st0, "cpu")
    for step in range(1, 11):
        g = torch.randn(n, generator=gen) * 1e-3
        expand_step(mine(), a, g.cuda(), step)
        expand_step(O, c, g, step)
    torch.cuda.synchronize()
    a = {k: v.cpu() for k, v in a.items()}
    dp = (a["p"] - c["p"]).abs()
    assert (dp <= 1e-5 * c["p"].abs() + 1e-8).float().mean() >= 0.995
    assert (dp <= 0.2 * HYPER["lr"]).all()
    for mom in ("m", "v"):
        same = a[f"k_{mom}"] == c[f"k_{mom}"]
        assert same.float().mean() >= 0.999
        for vec in ("s", "r"):
            x, y = a[f"{vec}_{mom}"][same], c[f"{vec}_{mom}"][same]
            # the group minimum is often an element whose update nearly cancels, so a last-place
            # difference in powf is amplified there (and carried along the ten steps): the reference's
            # own figure of 1e-4 on >= 99 % of the groups, 1e-2 on all
            assert ((x - y).abs() <= 1e-4 * y.abs()).float().mean() >= 0.99
            assert torch.allclose(x, y, rtol=1e-2)
        el = same.repeat_interleave(128)[:n]
        x, y = a[mom][el].to(torch.int16), c[mom][el].to(torch.int16)
        assert (x == y).float().mean() >= 0.995
        assert ((x - y).abs() <= 1).all()


def test_expand_golden_vectors_through_c_abi():
    """The reference's own expectation (pure PyTorch, generated on CPU from the reference checkout)
    against the CUDA kernel: weights and sqrt(max*min) everywhere, codes and scales on the groups
    where the test's table search and the kernel's closed form pick the same exponent."""
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "adamw_expand_golden.npz"))
    for name in sorted({k.split("/")[0] for k in z.files}):
        if name.startswith("ref_seed0"):
            continue  # NaN-ridden second moment, covered on the CPU side for the first moment only
        t = lambda k: torch.from_numpy(z[f"{name}/in/{k}"].copy()).cuda()
        h = lambda k: float(z[f"{name}/hyper/{k}"])
        e = lambda k: torch.from_numpy(z[f"{name}/out/{k}"])
        st = dict(p=t("params").flatten(), m=t("exp_avg").flatten(), v=t("exp_avg_sq").flatten(),
                  s_m=t("scale_exp_avg"), k_m=t("expand_exp_avg"), r_m=t("sqrtminmax_exp_avg"),
                  s_v=t("scale_exp_avg_sq"), k_v=t("expand_exp_avg_sq"), r_v=t("sqrtminmax_exp_avg_sq"))
        p_before = st["p"].cpu().clone()
        hyper = dict(beta1=h("beta1"), beta2=h("beta2"), lr=h("lr"), wd=h("wd"), eps=h("eps"))
        expand_step(mine(), st, t("grads").flatten(), int(h("step")), hyper=hyper)
        torch.cuda.synchronize()
        st = {k: v.cpu() for k, v in st.items()}

        def close(a, b):
            tight = (a - b).abs() <= 1e-8 + 1e-4 * b.abs()
            return tight.float().mean().item() >= 0.95 and torch.allclose(a, b, rtol=2e-3)

        assert ((e("params_py") - st["p"]).abs() <= 1e-4 * e("params_py").abs() + 1e-6 * p_before.abs()).all()
        for mom, sfx, exp_name in (("m", "", "B1Exp"), ("v", "_sq", "B2Exp")):
            n1 = "1" if mom == "m" else "2"
            assert close(e(f"block_sqrt_minmax{n1}"), st[f"r_{mom}"])
            same = e(exp_name) == st[f"k_{mom}"]
            assert same.float().mean() >= 0.5
            el = same.repeat_interleave(128)
            got = O.decode_fp8(st[mom]).to(torch.bfloat16).float()
            assert close(e(f"Qexp_avg{sfx}_py").to(torch.bfloat16).float()[el], got[el])
            assert close(e(f"Sexp_avg{sfx}_py")[same], st[f"s_{mom}"][same])


# ---------------------------------------------------------------------------------------------
# 3. the boundary itself
# ---------------------------------------------------------------------------------------------

def test_error_conventions():
    q = mine()
    n = 256
    st, _ = fresh(n)
    st = to(st, "cuda")
    g = torch.zeros(n, device="cuda")
    with pytest.raises(RuntimeError, match="128"):
        q.fp8_adamw_expand_step(st["p"], g, st["m"], st["s_m"], st["k_m"], st["r_m"], st["v"], st["s_v"],
                                st["k_v"], st["r_v"], 0.9, 0.95, 1e-4, 0.1, 1e-8, 1, 64, 16)
    with pytest.raises(RuntimeError):  # one scale per group
        q.fp8_adamw_expand_step(st["p"], g, st["m"], st["s_m"][:1], st["k_m"], st["r_m"], st["v"], st["s_v"],
                                st["k_v"], st["r_v"], 0.9, 0.95, 1e-4, 0.1, 1e-8, 1, 128, 16)
    with pytest.raises(RuntimeError, match="Float"):  # per-group vectors are read as float32
        q.fp8_adamw_expand_step(st["p"], g, st["m"], st["s_m"].bfloat16(), st["k_m"], st["r_m"], st["v"],
                                st["s_v"], st["k_v"], st["r_v"], 0.9, 0.95, 1e-4, 0.1, 1e-8, 1, 128, 16)
    with pytest.raises(RuntimeError, match="CUDA"):  # there is no CPU path
        q.fp8_adamw_expand_step(st["p"].cpu(), g, st["m"], st["s_m"], st["k_m"], st["r_m"], st["v"], st["s_v"],
                                st["k_v"], st["r_v"], 0.9, 0.95, 1e-4, 0.1, 1e-8, 1, 128, 16)
    # empty tensor: nothing to do, no error
    e = torch.empty(0, device="cuda")
    q.fp8_adamw_expand_step(e, e, e.to(torch.uint8), e, e, e, e.to(torch.uint8), e, e, e, 0.9, 0.95, 1e-4, 0.1,
                            1e-8, 1, 128, 16)


def test_unaligned_views_match_aligned():
    """A parameter that starts at an odd element offset (a slice of a flat buffer) takes the scalar
    access path and must give the same result as an aligned copy."""
    n = 128 * 9 + 17
    st0, gen = fresh(n, seed=8)
    g0 = torch.randn(n, generator=gen) * 1e-3
    a = to(st0, "cuda")
    big = {k: torch.zeros(v.numel() + 3, dtype=v.dtype, device="cuda") for k, v in st0.items()}
    b = {k: big[k][1:1 + v.numel()] for k, v in st0.items()}
    for k in b:
        b[k].copy_(st0[k])
    gb = torch.zeros(n + 3, device="cuda")[1:1 + n]
    gb.copy_(g0)
    for step in (1, 2, 3):
        expand_step(mine(), a, g0.cuda(), step)
        expand_step(mine(), b, gb, step)
    torch.cuda.synchronize()
    assert_bit_equal(a, b, keys=STATE_KEYS, what="unaligned view")
    assert_weights_close(a, b, HYPER["lr"], what="unaligned view")


def test_bf16_weight_copy():
    n = 128 * 20 + 1
    st0, gen = fresh(n, seed=9)
    a = to(st0, "cuda")
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    g = (torch.randn(n, generator=gen) * 1e-3).cuda()
    expand_step(mine(), a, g, 1, bf16_out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, a["p"].to(torch.bfloat16))
