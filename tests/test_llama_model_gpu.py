"""GPU tests of the model composition in training mode (FP8 activation stream through two decoder layers,
loss head, FP8 optimizer): loss and gradients against the same model evaluated without quantisation, and a
short training run.  Tolerances as derived in test_llama_layer_gpu.py (weight gradients carry E5M2 x E4M3
products whose gradient factor has crossed several E5M2 stages; with two layers the deepest ones cross up to
six): relative Frobenius error <= 0.2 and cosine >= 0.98 for weight gradients, loss within 1 %."""
from types import SimpleNamespace

import pytest
import torch

from coat_b200.fp8_trainer import MasterWeights, build_coat_optimizer
from coat_b200.models import CoatLlamaConfig, CoatLlamaForCausalLM
from coat_b200.utils._fp8manager import FP8Manager

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=256, intermediate_size=640, num_attention_heads=4, num_key_value_heads=4, vocab_size=512,
           num_hidden_layers=2, rms_norm_eps=1e-5, coat_fp8_args=dict(group_size=16))
B, S = 2, 128


def build(seed=11):
    torch.manual_seed(seed)
    model = CoatLlamaForCausalLM(CoatLlamaConfig(**CFG)).to("cuda", torch.bfloat16)
    ids = torch.randint(0, CFG["vocab_size"], (B, S), generator=torch.Generator().manual_seed(seed)).cuda()
    return model, ids


def test_training_loss_and_gradients_against_unquantised_model():
    model, ids = build()
    FP8Manager.is_first_microbatch = True
    model.train()
    loss = model(input_ids=ids, labels=ids).loss
    loss.backward()
    grads = {n: p.grad.detach().float().clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    ref = CoatLlamaForCausalLM(CoatLlamaConfig(**CFG)).to("cuda", torch.float32)
    ref.load_state_dict({k: v.float() for k, v in model.state_dict().items()})
    ref.eval()   # evaluation mode = the plain torch operators; autograd still works
    ref_loss = ref(input_ids=ids, labels=ids).loss
    ref_loss.backward()
    loss, ref_loss = float(loss.detach()), float(ref_loss.detach())
    assert abs(loss - ref_loss) <= 0.01 * ref_loss, (loss, ref_loss)
    for n, p in ref.named_parameters():
        t, r = grads[n].double().flatten(), p.grad.double().flatten()
        rel = float((t - r).norm() / r.norm())
        cos = float(torch.dot(t, r) / (t.norm() * r.norm()))
        assert rel <= 0.2 and cos >= 0.98, f"{n}: relative error {rel:.4f}, cosine {cos:.5f}"


def test_short_training_run_reduces_the_loss():
    model, ids = build(12)
    model.train()
    args = SimpleNamespace(learning_rate=2e-3, adam_beta1=0.9, adam_beta2=0.95, adam_epsilon=1e-8, weight_decay=0.0)
    decay = [n for n, p in model.named_parameters() if p.dim() == 2]
    masters = MasterWeights(model)   # fp32 masters: the optimizer steps them and writes the bf16 weights itself
    opt = build_coat_optimizer(masters, args, decay)
    masters.attach(opt)
    losses = []
    for _ in range(12):
        FP8Manager.is_first_microbatch = True
        loss = model(input_ids=ids, labels=ids).loss
        loss.backward()
        masters.copy_grads()
        opt.step()
        losses.append(float(loss.detach()))
    assert all(l == l for l in losses), losses
    assert losses[-1] < 0.6 * losses[0], losses
    for m, p in zip(masters.masters, masters.model_params):   # the fused bf16 copy is the rounded master
        assert torch.equal(p.detach(), m.detach().to(torch.bfloat16))


def test_stock_checkpoint_names_load():
    from coat_b200.models import make_state_dict_compatible
    model, ids = build(13)
    stock = {}
    for k, v in model.state_dict().items():
        for new, old in (("BeforeAttention.q_proj", "self_attn.q_proj"), ("BeforeAttention.k_proj", "self_attn.k_proj"),
                         ("BeforeAttention.v_proj", "self_attn.v_proj"), ("AfterAttention.o_proj", "self_attn.o_proj"),
                         ("MLPResidual.gate_proj", "mlp.gate_proj"), ("MLPResidual.up_proj", "mlp.up_proj"),
                         ("MLPResidual.down_proj", "mlp.down_proj")):
            k = k.replace(new, old)
        stock[k] = v.clone()
    other = CoatLlamaForCausalLM(CoatLlamaConfig(**CFG)).to("cuda", torch.bfloat16)
    other.load_state_dict(make_state_dict_compatible(stock), strict=True)
    model.eval(), other.eval()
    with torch.no_grad():
        assert torch.equal(model(input_ids=ids).logits, other(input_ids=ids).logits)
