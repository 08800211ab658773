"""GPU tests of the optimizer CLASS (coat_b200/optimizer/fp8_adamw.py): the state layout of the reference
(coat/optimizer/fp8_adamw.py:117-140), checkpoint round trips through its no-cast load_state_dict (:158-262),
the one-launch multi-tensor path against the per-tensor path, parameter groups, and the error conventions."""
import copy
import io

import pytest
import torch

from coat_b200.optimizer.fp8_adamw import CoatAdamW
from coat_b200.utils._fp8_quantization_config import QuantizationConfig

pytestmark = pytest.mark.gpu

SHAPES = [(256, 128), (1000,), (77, 3), (128,), (4096, 9)]   # full groups, ragged tails, one tiny tensor


def make(seed, **kw):
    gen = torch.Generator().manual_seed(seed)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).cuda()) for s in SHAPES]
    groups = [{"params": params[:3], "weight_decay": 0.1}, {"params": params[3:], "weight_decay": 0.0}]
    return params, CoatAdamW(groups, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, **kw)


def set_grads(params, seed):
    gen = torch.Generator().manual_seed(seed)
    for p in params:
        p.grad = (torch.randn(p.shape, generator=gen) * 1e-3).cuda()


def run(params, opt, steps, seed0=100):
    for t in range(steps):
        set_grads(params, seed0 + t)
        opt.step()


def same_state(a, b):
    sa, sb = a.state_dict()["state"], b.state_dict()["state"]
    assert sa.keys() == sb.keys()
    for k in sa:
        assert sa[k].keys() == sb[k].keys()
        for name in sa[k]:
            x, y = sa[k][name], sb[k][name]
            assert x.dtype == y.dtype and x.shape == y.shape, (k, name)
            if x.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
                x, y = x.view(torch.uint8), y.view(torch.uint8)
            assert torch.equal(x.cpu(), y.cpu()), (k, name)


def test_state_layout_matches_the_reference():
    params, opt = make(0)
    run(params, opt, 1)
    for p in params:
        st = opt.state[p]
        groups = (p.numel() + 127) // 128
        assert list(st.keys()) == ["step", "exp_avg", "scale_exp_avg", "expand_exp_avg", "sqrt_minmax_exp_avg",
                                   "exp_avg_sq", "scale_exp_avg_sq", "expand_exp_avg_sq", "sqrt_minmax_exp_avg_sq"]
        assert st["step"].device.type == "cpu" and float(st["step"]) == 1.0
        for k in ("exp_avg", "exp_avg_sq"):
            assert st[k].dtype == torch.float8_e4m3fn and st[k].shape == p.shape and st[k].is_cuda
        for k in ("scale_exp_avg", "expand_exp_avg", "sqrt_minmax_exp_avg", "scale_exp_avg_sq", "expand_exp_avg_sq",
                  "sqrt_minmax_exp_avg_sq"):
            assert st[k].dtype == torch.float32 and st[k].shape == (groups,)


def test_no_expansion_keeps_only_scales():
    q = QuantizationConfig(first_order_expansion="false", second_order_expansion="false")
    params, opt = make(1, qargs=q)
    run(params, opt, 2)
    assert "expand_exp_avg" not in opt.state[params[0]] and "scale_exp_avg_sq" in opt.state[params[0]]


@pytest.mark.parametrize("through_cpu_file", [False, True])
def test_checkpoint_round_trip_continues_bit_for_bit(through_cpu_file):
    pa, oa = make(2)
    run(pa, oa, 3)
    sd = oa.state_dict()
    if through_cpu_file:   # torch.save / torch.load with map_location="cpu", as a trainer would
        buf = io.BytesIO()
        torch.save(sd, buf)
        buf.seek(0)
        sd = torch.load(buf, map_location="cpu", weights_only=False)
        assert sd["state"][0]["exp_avg"].dtype == torch.float8_e4m3fn and not sd["state"][0]["exp_avg"].is_cuda
    else:
        sd = copy.deepcopy(sd)
    pb, ob = make(2)
    with torch.no_grad():
        for a, b in zip(pa, pb):
            b.copy_(a)
    ob.load_state_dict(sd)
    for p in pb:   # moved to the parameter's device, dtype untouched (the stock loader would cast the codes to fp32)
        assert ob.state[p]["exp_avg"].dtype == torch.float8_e4m3fn and ob.state[p]["exp_avg"].is_cuda
        assert ob.state[p]["scale_exp_avg"].dtype == torch.float32 and float(ob.state[p]["step"]) == 3.0
    run(pa, oa, 3, seed0=200)
    run(pb, ob, 3, seed0=200)
    for a, b in zip(pa, pb):
        assert torch.equal(a, b)
    same_state(oa, ob)


def test_multi_tensor_launch_equals_per_tensor_launches():
    pa, oa = make(3, multi_tensor=True)
    pb, ob = make(3, multi_tensor=False)
    run(pa, oa, 4)
    run(pb, ob, 4)
    for a, b in zip(pa, pb):
        assert torch.equal(a, b)
    same_state(oa, ob)


def test_parameter_groups_use_their_own_weight_decay_and_lr():
    pa, oa = make(4)
    pb, ob = make(4)
    ob.param_groups[1]["weight_decay"] = 0.5
    ob.param_groups[1]["lr"] = 5e-3
    run(pa, oa, 2)
    run(pb, ob, 2)
    assert all(torch.equal(a, b) for a, b in zip(pa[:3], pb[:3]))
    assert all(not torch.equal(a, b) for a, b in zip(pa[3:], pb[3:]))


def test_parameters_without_gradient_are_skipped():
    params, opt = make(5)
    before = [p.detach().clone() for p in params]
    set_grads(params, 1)
    params[1].grad = None
    opt.step()
    assert torch.equal(params[1], before[1]) and len(opt.state[params[1]]) == 0
    assert not torch.equal(params[0], before[0])


def test_error_conventions():
    p = torch.nn.Parameter(torch.zeros(256, device="cuda", dtype=torch.bfloat16))
    opt = CoatAdamW([p])
    p.grad = torch.zeros_like(p)
    with pytest.raises(RuntimeError):
        opt.step()
    with pytest.raises(ValueError):
        CoatAdamW([torch.nn.Parameter(torch.zeros(4, device="cuda"))], lr=-1.0)
    with pytest.raises(AssertionError):
        CoatAdamW([torch.nn.Parameter(torch.zeros(4, device="cuda"))],
                  qargs=QuantizationConfig(first_order_expansion="true", second_order_expansion="false"))
    q = torch.nn.Parameter(torch.zeros(256, device="cuda"))
    opt = CoatAdamW([q], amsgrad=True)
    q.grad = torch.zeros_like(q)
    with pytest.raises(RuntimeError):
        opt.step()


def test_fused_bf16_copy_of_master_weights():
    params, opt = make(6)
    copies = [torch.zeros(p.numel(), dtype=torch.bfloat16, device="cuda") for p in params]
    opt.attach_bf16_weights(zip(params, copies))
    run(params, opt, 2)
    for p, c in zip(params, copies):
        assert torch.equal(c, p.detach().flatten().to(torch.bfloat16))
    with pytest.raises(ValueError):
        opt.attach_bf16_weights([(params[0], torch.zeros(3, dtype=torch.bfloat16, device="cuda"))])


# ------------------------------------------------------------------------------------------------------
# interchange with the REFERENCE's optimizer class (its python class on its own compiled kernels)
# ------------------------------------------------------------------------------------------------------
INTERCHANGE_SHAPES = [(256, 128), (1000,), (77, 3), (128,), (4096, 9), (512, 512)]


def _pair(seed, qargs_kw):
    """The same parameters twice: one set for the reference's CoatAdamW, one for this repository's."""
    from _ref import load_ref_optimizer
    ref = load_ref_optimizer()
    if ref is None:
        pytest.skip("the reference's optimizer class is not staged (python oracle/build_ref.py)")
    RefAdamW, RefConfig = ref
    gen = torch.Generator().manual_seed(seed)
    init = [torch.randn(s, generator=gen) * 0.02 for s in INTERCHANGE_SHAPES]
    pr = [torch.nn.Parameter(t.clone().cuda()) for t in init]
    pm = [torch.nn.Parameter(t.clone().cuda()) for t in init]
    hyper = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    return pr, RefAdamW(pr, qargs=RefConfig(**qargs_kw), **hyper), pm, (lambda: CoatAdamW(pm, qargs=QuantizationConfig(**qargs_kw), **hyper))


@pytest.mark.parametrize("expansion", ["true", "false"])
def test_state_dict_written_by_the_reference_class_loads_and_continues_bit_for_bit(expansion):
    """Three steps with the reference's own CoatAdamW (its class, its compiled kernels), its state_dict saved with
    torch.save, loaded into this repository's CoatAdamW, then both continue for three more steps on the same
    gradients: keys, dtypes and shapes of the state as the reference wrote them; after the continuation every
    quantised state array bit-identical, weights bit-identical in exact mode and within the stated tolerance of the
    default mode."""
    from coat_b200 import _lib
    kw = dict(first_order_expansion=expansion, second_order_expansion=expansion)
    pr, ref_opt, pm, make_mine = _pair(31, kw)
    run(pr, ref_opt, 3)
    buf = io.BytesIO()
    torch.save(ref_opt.state_dict(), buf)
    buf.seek(0)
    sd = torch.load(buf, map_location="cpu", weights_only=False)
    with torch.no_grad():
        for a, b in zip(pr, pm):
            b.copy_(a)
    for exact in (True, False):
        with torch.no_grad():
            start = [p.detach().clone() for p in pr]
        mine = make_mine()
        mine.load_state_dict(copy.deepcopy(sd))
        for p in pm:
            st = mine.state[p]
            assert st["exp_avg"].dtype == torch.float8_e4m3fn and st["exp_avg"].is_cuda and float(st["step"]) == 3.0
            assert st["scale_exp_avg"].dtype == torch.float32
        ref_sd = copy.deepcopy(ref_opt.state_dict())
        old_flags = getattr(mine, "kernel_flags", None)
        if exact:
            mine.kernel_flags = _lib.ADAMW_EXACT_POW
        run(pr, ref_opt, 3, seed0=300)
        run(pm, mine, 3, seed0=300)
        same_state(ref_opt, mine)
        for a, b in zip(pr, pm):
            if exact:
                assert torch.equal(a, b)
            else:
                assert bool(((a - b).abs() <= 2.4e-7 * a.abs() + 1e-5 * 1e-3 * 10 * 3).all())
        # rewind both for the second mode
        ref_opt.load_state_dict(ref_sd)
        with torch.no_grad():
            for p, s0, q in zip(pr, start, pm):
                p.copy_(s0)
                q.copy_(s0)
        del old_flags
