"""CPU tests of the model composition (coat_b200/models/coat_llama_model.py): checkpoint key renaming, and the
evaluation-mode forward (plain bf16/fp32 torch operators, no FP8 stream) against a stack of unquantised
reference layers (oracle/llama_layer.py).  The FP8 training path is tested on the GPU in
test_llama_model_gpu.py."""
import torch
import torch.nn.functional as F

from coat_b200.models import CoatLlamaConfig, CoatLlamaForCausalLM, chunked_causal_lm_loss, make_state_dict_compatible
from oracle.llama_layer import reference_layer

CFG = dict(hidden_size=64, intermediate_size=128, num_attention_heads=4, num_key_value_heads=2, vocab_size=97,
           num_hidden_layers=2, rms_norm_eps=1e-5, coat_fp8_args=dict(group_size=16))


def stock_names(model):
    """The model's state dict under the key names of a stock Llama checkpoint."""
    back = {"BeforeAttention.q_proj": "self_attn.q_proj", "BeforeAttention.k_proj": "self_attn.k_proj",
            "BeforeAttention.v_proj": "self_attn.v_proj", "AfterAttention.o_proj": "self_attn.o_proj",
            "MLPResidual.gate_proj": "mlp.gate_proj", "MLPResidual.up_proj": "mlp.up_proj",
            "MLPResidual.down_proj": "mlp.down_proj"}
    out = {}
    for k, v in model.state_dict().items():
        for new, old in back.items():
            k = k.replace(new, old)
        out[k] = v.clone()
    return out


def test_state_dict_renaming_round_trip():
    torch.manual_seed(0)
    a, b = CoatLlamaForCausalLM(CoatLlamaConfig(**CFG)), CoatLlamaForCausalLM(CoatLlamaConfig(**CFG))
    stock = stock_names(a)
    assert "model.layers.1.self_attn.o_proj.weight" in stock and "model.layers.0.mlp.up_proj.weight" in stock
    assert not any("BeforeAttention" in k or "MLPResidual" in k or "AfterAttention" in k for k in stock)
    renamed = make_state_dict_compatible(stock)
    assert set(renamed) == set(b.state_dict())
    missing, unexpected = b.load_state_dict(renamed, strict=True)
    assert not missing and not unexpected
    for (ka, va), (kb, vb) in zip(a.state_dict().items(), b.state_dict().items()):
        assert ka == kb and torch.equal(va, vb)
    # already-renamed keys pass unchanged
    assert make_state_dict_compatible(renamed).keys() == renamed.keys()


def test_eval_forward_matches_reference_layers():
    torch.manual_seed(1)
    cfg = CoatLlamaConfig(**CFG)
    model = CoatLlamaForCausalLM(cfg).double().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "layernorm" in name or name.endswith("norm.weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
    ids = torch.randint(0, cfg.vocab_size, (2, 24))
    with torch.no_grad():
        out = model(input_ids=ids, labels=ids, return_logits=True)
        x = model.model.embed_tokens(ids)
        for layer in model.model.layers:
            w = {"q": layer.BeforeAttention.q_proj.weight, "k": layer.BeforeAttention.k_proj.weight,
                 "v": layer.BeforeAttention.v_proj.weight, "o": layer.AfterAttention.o_proj.weight,
                 "gate": layer.MLPResidual.gate_proj.weight, "up": layer.MLPResidual.up_proj.weight,
                 "down": layer.MLPResidual.down_proj.weight, "ln1": layer.input_layernorm.weight,
                 "ln2": layer.post_attention_layernorm.weight}
            x = reference_layer(x, w, cfg.num_attention_heads, cfg.num_key_value_heads, eps=torch.finfo(torch.float64).eps)
        x = F.rms_norm(x, (cfg.hidden_size,), model.model.norm.weight, cfg.rms_norm_eps)
        logits = x @ model.lm_head.weight.t()
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, cfg.vocab_size), ids[:, 1:].reshape(-1))
    assert torch.allclose(out.logits, logits, rtol=1e-9, atol=1e-9)
    assert abs(float(out.loss) - float(loss)) < 2e-6   # the loss is accumulated in fp32


def test_padding_mask_matches_unpadded_prefix():
    torch.manual_seed(2)
    cfg = CoatLlamaConfig(**CFG)
    model = CoatLlamaForCausalLM(cfg).double().eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 16))
    mask = torch.ones(1, 16, dtype=torch.long)
    mask[0, 12:] = 0
    with torch.no_grad():
        padded = model(input_ids=ids, attention_mask=mask).logits[:, :12]
        short = model(input_ids=ids[:, :12]).logits
    assert torch.allclose(padded, short, rtol=1e-9, atol=1e-9)


def test_chunked_loss_equals_plain_loss_and_ignores_labels():
    torch.manual_seed(3)
    h = torch.randn(2, 9, 16, dtype=torch.float64, requires_grad=True)
    w = torch.randn(31, 16, dtype=torch.float64, requires_grad=True)
    y = torch.randint(0, 31, (2, 9))
    y[0, 3] = -100
    plain = F.cross_entropy((h[:, :-1] @ w.t()).reshape(-1, 31), y[:, 1:].reshape(-1), ignore_index=-100)
    chunked = chunked_causal_lm_loss(h, w, y, chunk_rows=5)
    assert abs(float(plain) - float(chunked)) < 2e-6   # fp32 logits inside
    gp = torch.autograd.grad(plain, (h, w))
    gc = torch.autograd.grad(chunked, (h, w))
    assert all(torch.allclose(a, b, atol=1e-6) for a, b in zip(gp, gc))
