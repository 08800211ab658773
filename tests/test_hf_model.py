"""The transformers-facing classes (coat_b200/models/hf.py) on the CPU: registration with the Auto classes, conversion
of a stock Llama checkpoint (coat/models/coat_llama_convert_from_hf.py:20-62 of the reference), save / load round trip,
and evaluation-mode logits equal to the stock model's.

The blocks' evaluation path normalises with `F.rms_norm(x, shape, weight)` and no epsilon, as the reference's does
(coat/models/coat_llama.py:217, 594), i.e. with torch's default (machine epsilon) instead of `config.rms_norm_eps`; the
stock model is therefore built with that epsilon, which makes the two models the same function."""
import pytest
import torch

transformers = pytest.importorskip("transformers")


def _stock(eps):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_attention_heads=4, num_key_value_heads=2,
                      num_hidden_layers=2, vocab_size=320, max_position_embeddings=64, rms_norm_eps=eps)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def test_convert_save_load_and_logits(tmp_path):
    from transformers import AutoConfig, AutoModelForCausalLM

    from coat_b200.models.hf import CoatLlamaConfig, CoatLlamaForCausalLM, ConvertArguments, download_and_convert_llama
    from coat_b200.utils._fp8_quantization_config import QuantizationConfig
    stock = _stock(torch.finfo(torch.float32).eps)
    stock.save_pretrained(tmp_path / "stock")
    download_and_convert_llama(ConvertArguments(str(tmp_path / "stock"), str(tmp_path / "coat")),
                               QuantizationConfig(group_size=16, weight_memory_efficient=True))
    cfg = AutoConfig.from_pretrained(tmp_path / "coat")
    assert isinstance(cfg, CoatLlamaConfig) and cfg.model_type == "fp8_llama"
    assert cfg.coat_fp8_args["group_size"] == 16 and cfg.coat_fp8_args["weight_memory_efficient"] is True
    model = AutoModelForCausalLM.from_pretrained(tmp_path / "coat").eval()
    assert isinstance(model, CoatLlamaForCausalLM)
    keys = set(model.state_dict())
    assert "model.layers.1.BeforeAttention.q_proj.weight" in keys and "model.layers.0.MLPResidual.down_proj.weight" in keys
    assert not any("self_attn" in k or ".mlp." in k for k in keys)
    ids = torch.randint(0, 320, (2, 24), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = stock(ids).logits
        got = model(ids).logits
        loss = model(ids, labels=ids).loss
        want_loss = stock(ids, labels=ids).loss
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(loss, want_loss, rtol=1e-5, atol=1e-6)


def test_from_config_initialises_and_plain_model_loads_the_same_checkpoint(tmp_path):
    from transformers import AutoModelForCausalLM

    from coat_b200.models import CoatLlamaForCausalLM as PlainCausalLM
    from coat_b200.models.hf import CoatLlamaConfig
    cfg = CoatLlamaConfig(hidden_size=128, intermediate_size=256, num_attention_heads=4, num_hidden_layers=1,
                          vocab_size=64, coat_fp8_args={"group_size": 16})
    torch.manual_seed(3)
    model = AutoModelForCausalLM.from_config(cfg)
    w = model.model.layers[0].MLPResidual.up_proj.weight
    assert 0.01 < float(w.detach().std()) < 0.03                      # initializer_range 0.02
    assert torch.equal(model.model.norm.weight, torch.ones(128))
    model.save_pretrained(tmp_path / "m")
    # the module tree and the state-dict keys are those of the plain nn.Module classes
    plain = PlainCausalLM(cfg)
    from safetensors.torch import load_file
    missing, unexpected = plain.load_state_dict(load_file(str(tmp_path / "m" / "model.safetensors")), strict=False)
    assert not unexpected and not missing
