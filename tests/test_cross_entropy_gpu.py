"""GPU tests of the cross-entropy loss head (coat_b200/activation/liger/cross_entropy.py on csrc/cross_entropy.cu)
against torch's cross_entropy with autograd and, where it is staged, against the reference's own Liger Triton kernel
(coat/activation/liger/cross_entropy.py) on the same logits.  fp32 arithmetic with approximate exponentials on both
GPU sides: tolerance 2e-5 relative on the loss, 2e-6 absolute on the gradients (softmax values are <= 1)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def data(rows, V, seed, dtype=torch.float32, ignore_every=5):
    gen = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, V, generator=gen) * 3).to(dtype).cuda()
    y = torch.randint(0, V, (rows,), generator=gen)
    if ignore_every:
        y[::ignore_every] = -100
    return x, y.cuda()


@pytest.mark.parametrize("rows,V", [(7, 1000), (64, 32000), (33, 32003), (4, 17)])
@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_against_torch(rows, V, reduction):
    from coat_b200.activation.liger import LigerCrossEntropyFunction
    x, y = data(rows, V, 1)
    xr = x.clone().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(xr, y, ignore_index=-100, reduction=reduction)
    xm = x.clone().requires_grad_(True)
    loss, z = LigerCrossEntropyFunction.apply(xm.clone(), y, -100, 0.0, 0.0, reduction)   # the clone is overwritten
    assert z is None
    assert torch.allclose(loss, ref, rtol=2e-5, atol=1e-6)
    w = torch.randn_like(ref)
    (ref * w).sum().backward()
    xm2 = x.clone().requires_grad_(True)
    loss2, _ = LigerCrossEntropyFunction.apply(xm2 * 1.0, y, -100, 0.0, 0.0, reduction)
    (loss2 * w).sum().backward()
    assert torch.allclose(xm2.grad, xr.grad, rtol=1e-4, atol=2e-6 * float(w.abs().max()))
    assert bool((xm2.grad[y == -100] == 0).all())


def test_bf16_logits_and_causal_lm_loss():
    from coat_b200.activation.liger import LigerForCausalLMLoss, liger_fixed_cross_entropy
    x, y = data(48, 4096, 2, dtype=torch.bfloat16)
    ref = torch.nn.functional.cross_entropy(x.float(), y, ignore_index=-100)
    got = liger_fixed_cross_entropy(x.clone(), y)
    assert got.dtype == torch.bfloat16 and abs(float(got) - float(ref)) <= 1e-2 * float(ref)
    B, S, V = 2, 24, 512
    gen = torch.Generator().manual_seed(3)
    logits = torch.randn(B, S, V, generator=gen).cuda().requires_grad_(True)
    labels = torch.randint(0, V, (B, S), generator=gen).cuda()
    labels[0, :5] = -100
    loss = LigerForCausalLMLoss(logits, labels, V)
    ref = torch.nn.functional.cross_entropy(logits.detach()[:, :-1].reshape(-1, V), labels[:, 1:].reshape(-1), ignore_index=-100)
    assert torch.allclose(loss, ref, rtol=2e-5)
    loss.backward()
    l2 = logits.detach().clone().requires_grad_(True)
    torch.nn.functional.cross_entropy(l2[:, :-1].reshape(-1, V), labels[:, 1:].reshape(-1), ignore_index=-100).backward()
    assert torch.allclose(logits.grad, l2.grad, rtol=1e-4, atol=2e-7)
    n = int((labels[:, 1:] != -100).sum())
    summed = LigerForCausalLMLoss(logits.detach(), labels, V, num_items_in_batch=n)
    assert torch.allclose(summed, ref, rtol=2e-5)


def test_unsupported_options_raise():
    from coat_b200.activation.liger import LigerCrossEntropyFunction
    x, y = data(4, 64, 4)
    with pytest.raises(NotImplementedError):
        LigerCrossEntropyFunction.apply(x, y, -100, 0.0, 0.1, "mean")
    with pytest.raises(RuntimeError):
        LigerCrossEntropyFunction.apply(x.cpu(), y.cpu(), -100, 0.0, 0.0, "mean")


@pytest.mark.parametrize("reduction", ["mean", "sum"])
def test_against_the_reference_liger_kernel(reduction):
    from oracle.ref_loader import load_ref_liger
    ref_mod = load_ref_liger()
    if ref_mod is None:
        pytest.skip("oracle/_ref/coat_ref/activation/liger not staged (python oracle/build_ref.py)")
    from coat_b200.activation.liger import cross_entropy as mine
    x, y = data(256, 32000, 5)
    a, b = x.clone(), x.clone()
    loss_r, _, grad_r = ref_mod.cross_entropy_forward(a, y, -100, 0.0, 0.0, reduction, None, False)
    loss_m, _, grad_m = mine.cross_entropy_forward(b, y, -100, 0.0, 0.0, reduction, None, False)
    print(f"PARITY liger cross entropy[{reduction}]: loss {float(loss_m):.6f} vs {float(loss_r):.6f}, "
          f"max gradient difference {float((grad_m - grad_r).abs().max()):.3e}")
    assert torch.allclose(loss_m, loss_r, rtol=2e-5)
    scale = 1.0 if reduction == "sum" else 1.0 / int((y != -100).sum())
    assert float((grad_m - grad_r).abs().max()) <= 2e-6 * scale
