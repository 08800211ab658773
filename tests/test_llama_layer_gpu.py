"""GPU test of the decoder-layer composition (coat_b200/models/coat_llama.py) against an unquantised
torch layer with autograd (oracle/llama_layer.py).

Tolerances, derived from the formats.  Rounding to E4M3 (3 mantissa bits) leaves an rms relative error of
0.0722 * sqrt(1/2) / 2 = 2.6 % per element, rounding to E5M2 (2 mantissa bits) 5.1 %.  Independent errors
average out over a GEMM's reduction only as far as the exact terms do, so a product of an E5M2 gradient
and an E4M3 activation carries ~5.7 %, and an error already present in a gradient is passed on in full:
  * the layer update y - x and the input gradient pass 3-5 quantisation points, mostly E4M3 or averaged by
    a reduction:                     relative Frobenius error <= 0.10, cosine similarity >= 0.995;
  * weight gradients are sums over tokens of E5M2 x E4M3 products whose E5M2 factor has itself come
    through up to three E5M2 stages (5.1 % * sqrt(3) = 8.8 %, plus the 5.7 % of the product: ~10.5 % for
    the deepest ones, q/k/v):        relative Frobenius error <= 0.15, cosine similarity >= 0.99.
The two weight-memory modes must agree bit for bit with each other (same codes, different caching)."""
import pytest
import torch

from coat_b200.activation.real_quantization.func_quantize import Coat_quantize_bgn, Coat_quantize_end
from coat_b200.models.coat_llama import CoatLlamaConfig, CoatLlamaDecoderLayer
from coat_b200.utils._fp8_quantization_config import QuantizationConfig
from coat_b200.utils._fp8manager import FP8Manager
from oracle.llama_layer import reference_layer

pytestmark = pytest.mark.gpu

H, I, HEADS, B, S = 512, 1408, 8, 2, 256   # head_dim 64; every dimension a multiple of 128


def build(memory_efficient, kv_heads=HEADS, seed=3):
    qargs = dict(group_size=16, weight_memory_efficient=memory_efficient)
    cfg = CoatLlamaConfig(hidden_size=H, intermediate_size=I, num_attention_heads=HEADS, num_key_value_heads=kv_heads,
                          rms_norm_eps=1e-5, coat_fp8_args=qargs)
    gen = torch.Generator().manual_seed(seed)
    layer = CoatLlamaDecoderLayer(cfg, 0)
    with torch.no_grad():
        for name, p in layer.named_parameters():
            if p.dim() == 2:
                p.copy_(torch.randn(p.shape, generator=gen) * 0.02)
            else:
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=gen))
    layer = layer.to("cuda", torch.bfloat16).train()
    x = (torch.randn(B, S, H, generator=gen) * 0.5).to(torch.bfloat16).cuda().requires_grad_(True)
    up = (torch.randn(B, S, H, generator=gen) * 1e-2).to(torch.bfloat16).cuda()
    return layer, QuantizationConfig(**qargs), x, up


def run(layer, qargs, x, up):
    FP8Manager.is_first_microbatch = True
    bgn, end = Coat_quantize_bgn(qargs).train(), Coat_quantize_end(qargs).train()
    (h, qh, sh), = layer(*bgn(x))
    y = end(h, qh, sh)
    y.backward(up)
    grads = {n: p.grad.detach().clone() for n, p in layer.named_parameters()}
    return y.detach(), x.grad.detach().clone(), grads


def weights_of(layer, dtype):
    g = lambda m: m.weight.detach().to(dtype).requires_grad_(True)
    return {"q": g(layer.BeforeAttention.q_proj), "k": g(layer.BeforeAttention.k_proj),
            "v": g(layer.BeforeAttention.v_proj), "o": g(layer.AfterAttention.o_proj),
            "gate": g(layer.MLPResidual.gate_proj), "up": g(layer.MLPResidual.up_proj),
            "down": g(layer.MLPResidual.down_proj), "ln1": g(layer.input_layernorm),
            "ln2": g(layer.post_attention_layernorm)}


NAMES = {"q": "BeforeAttention.q_proj.weight", "k": "BeforeAttention.k_proj.weight",
         "v": "BeforeAttention.v_proj.weight", "o": "AfterAttention.o_proj.weight",
         "gate": "MLPResidual.gate_proj.weight", "up": "MLPResidual.up_proj.weight",
         "down": "MLPResidual.down_proj.weight", "ln1": "input_layernorm.weight",
         "ln2": "post_attention_layernorm.weight"}


def close(t, r, what, max_rel=0.10, min_cos=0.995):
    t, r = t.double().flatten(), r.double().flatten()
    rel = float((t - r).norm() / r.norm())
    cos = float(torch.dot(t, r) / (t.norm() * r.norm()))
    assert rel <= max_rel and cos >= min_cos, f"{what}: relative error {rel:.4f}, cosine {cos:.5f}"


@pytest.mark.parametrize("kv_heads", [HEADS, 2])
def test_layer_forward_backward_against_unquantised_layer(kv_heads):
    layer, qargs, x, up = build(True, kv_heads)
    y, dx, grads = run(layer, qargs, x, up)
    w = weights_of(layer, torch.float32)
    xr = x.detach().float().requires_grad_(True)
    yr = reference_layer(xr, w, HEADS, kv_heads)
    yr.backward(up.float())
    close(y.float() - x.detach().float(), yr.detach() - xr.detach(), "layer update")
    close(dx, xr.grad, "input gradient")
    for short, name in NAMES.items():
        close(grads[name], w[short].grad, f"gradient of {name}", max_rel=0.15, min_cos=0.99)


def test_cached_weights_equal_memory_efficient_mode():
    a = run(*build(True))
    b = run(*build(False))
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    for n in a[2]:
        assert torch.equal(a[2][n], b[2][n]), n


def test_second_microbatch_reuses_cached_scales():
    layer, qargs, x, up = build(True)
    y1, dx1, _ = run(layer, qargs, x, up)
    layer.zero_grad(set_to_none=True)
    x.grad = None
    FP8Manager.is_first_microbatch = False
    bgn, end = Coat_quantize_bgn(qargs).train(), Coat_quantize_end(qargs).train()
    (h, qh, sh), = layer(*bgn(x))
    y2 = end(h, qh, sh)
    y2.backward(up)
    FP8Manager.is_first_microbatch = True
    assert torch.equal(y1, y2.detach()) and torch.equal(dx1, x.grad)


def test_eval_mode_is_the_plain_bf16_layer():
    layer, qargs, x, up = build(True)
    layer.eval()
    with torch.no_grad():
        (h, qh, sh), = layer(x.detach(), None, None)
    assert qh is None and sh is None
    yr = reference_layer(x.detach().float(), {k: v.detach() for k, v in weights_of(layer, torch.float32).items()},
                         HEADS, HEADS, eps=torch.finfo(torch.bfloat16).eps)
    close(h.float() - x.detach().float(), yr - x.detach().float(), "eval-mode update")


def test_fused_rotary_matches_the_eager_form():
    """One rounding to bf16 instead of one per operation: within 2 bf16 ulps of the eager result, and the
    backward kernel is the exact transpose (checked against autograd of the eager form in fp32)."""
    from coat_b200.models.coat_llama import _FusedRotary, _rotate_half, llama_rotary_embeddings
    gen = torch.Generator().manual_seed(21)
    B, S, Hh, D = 2, 96, 4, 64
    x = torch.randn(B, S, Hh, D, generator=gen).to(torch.bfloat16).cuda()
    dy = torch.randn(B, Hh, S, D, generator=gen).to(torch.bfloat16).cuda().transpose(1, 2)   # a transposed view
    cos, sin = llama_rotary_embeddings(torch.arange(S, device="cuda")[None, :], D, 10000.0, torch.bfloat16)
    xg = x.clone().requires_grad_(True)
    y = _FusedRotary.apply(xg, cos, sin)
    y.backward(dy)
    xr = x.float().requires_grad_(True)
    c, s = cos.float().unsqueeze(2), sin.float().unsqueeze(2)
    yr = xr * c + _rotate_half(xr) * s
    yr.backward(dy.float())
    ulp = lambda t: torch.exp2(torch.floor(torch.log2(t.abs().clamp_min(1e-30))) - 7)
    assert bool(((y.float() - yr.detach()).abs() <= 2 * ulp(yr.detach()) + 1e-6).all())
    assert bool(((xg.grad.float() - xr.grad).abs() <= 2 * ulp(xr.grad) + 1e-6).all())
