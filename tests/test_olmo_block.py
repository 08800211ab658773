"""Host-side checks of the OLMo block (no GPU): parameter names as the reference's block registers them
(coat/models/coat_olmo.py:112,264,398-404: `BeforeAttention.att_proj`, `AfterAttention.attn_out`, `MLPResidual.ff_proj`,
`MLPResidual.ff_out`), evaluation mode equal to the unquantised block, configurations the block refuses."""
import pytest
import torch

from coat_b200.models.coat_olmo import CoatOLMoBlock, CoatOLMoConfig, CoatOLMoSequentialBlock
from coat_b200.utils._fp8_quantization_config import QuantizationConfig
from oracle.olmo_block import reference_block


def test_parameter_names_and_eval_forward():
    cfg = CoatOLMoConfig(d_model=128, n_heads=4, mlp_hidden_size=512, max_sequence_length=16)
    block = CoatOLMoBlock.build(3, cfg, QuantizationConfig(group_size=16))
    assert isinstance(block, CoatOLMoSequentialBlock)
    torch.manual_seed(0)
    block.reset_parameters()
    names = [n for n, _ in block.named_parameters()]
    assert names == ["BeforeAttention.att_proj.weight", "AfterAttention.attn_out.weight", "MLPResidual.ff_proj.weight",
                     "MLPResidual.ff_out.weight"]
    assert block.MLPResidual.ff_proj.weight.shape == (512, 128) and block.MLPResidual.ff_out.weight.shape == (128, 256)
    # mitchell initialisation: the output projections shrink with the layer index
    assert float(block.AfterAttention.attn_out.weight.std()) < float(block.BeforeAttention.att_proj.weight.std())
    block.eval()
    x = torch.randn(2, 16, 128)
    with torch.no_grad():
        y, qx, sx, cache = block(x, None, None)
    w = {"att_proj": block.BeforeAttention.att_proj.weight, "attn_out": block.AfterAttention.attn_out.weight,
         "ff_proj": block.MLPResidual.ff_proj.weight, "ff_out": block.MLPResidual.ff_out.weight}
    assert qx is None and sx is None and cache is None
    torch.testing.assert_close(y, reference_block(x, w, 4), rtol=1e-4, atol=1e-5)


def test_grouped_query_dimensions():
    cfg = CoatOLMoConfig(d_model=128, n_heads=8, n_kv_heads=2, mlp_hidden_size=512)
    block = CoatOLMoSequentialBlock(0, cfg, QuantizationConfig(group_size=16))
    assert block.fused_dims == (128, 32, 32) and block.BeforeAttention.att_proj.weight.shape == (192, 128)


@pytest.mark.parametrize("kw", [dict(activation_type="gelu"), dict(layer_norm_with_affine=True), dict(include_bias=True),
                                dict(norm_after=True), dict(attention_layer_norm=True)])
def test_unsupported_configurations_are_refused(kw):
    with pytest.raises((NotImplementedError, AssertionError)):
        CoatOLMoSequentialBlock(0, CoatOLMoConfig(d_model=128, n_heads=4, mlp_hidden_size=512, **kw),
                                QuantizationConfig(group_size=16))


def test_whole_model_eval_forward_masks_and_keys():
    from coat_b200.models.coat_olmo import CoatOLMo
    cfg = CoatOLMoConfig(d_model=128, n_heads=4, n_layers=2, mlp_hidden_size=512, vocab_size=100, embedding_size=128,
                         max_sequence_length=32, weight_tying=False)
    torch.manual_seed(0)
    model = CoatOLMo(cfg, QuantizationConfig(group_size=16)).eval()
    keys = list(model.state_dict())
    assert keys[0] == "transformer.wte.weight" and "transformer.ff_out.weight" in keys
    assert "transformer.blocks.1.MLPResidual.ff_proj.weight" in keys
    ids = torch.randint(0, 100, (2, 16), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        out = model(ids, output_hidden_states=True)
        x = model.transformer.wte(ids)
        for b in model.transformer.blocks:
            w = {"att_proj": b.BeforeAttention.att_proj.weight, "attn_out": b.AfterAttention.attn_out.weight,
                 "ff_proj": b.MLPResidual.ff_proj.weight, "ff_out": b.MLPResidual.ff_out.weight}
            x = reference_block(x, w, 4)
        want = model.transformer.ff_out(torch.nn.functional.layer_norm(x, (128,)))
        torch.testing.assert_close(out.logits, want, rtol=1e-4, atol=1e-5)
        assert len(out.hidden_states) == 3 and out.attn_key_values is None
        # a padding mask changes nothing before the padding (causal attention) and nothing in unpadded sequences
        mask = torch.ones(2, 16)
        mask[1, 10:] = 0
        masked = model(ids, attention_mask=mask).logits
        torch.testing.assert_close(masked[0], out.logits[0])
        torch.testing.assert_close(masked[1, :10], out.logits[1, :10])
        assert model(ids, last_logits_only=True).logits.shape == (2, 1, 128)
    tied = CoatOLMo(CoatOLMoConfig(d_model=128, n_heads=4, n_layers=1, mlp_hidden_size=512, vocab_size=64,
                                   weight_tying=True), QuantizationConfig(group_size=16))
    tied.eval()   # (training mode needs the CUDA kernels)
    with torch.no_grad():
        assert "ff_out" not in tied.transformer and tied(ids % 64).logits.shape == (2, 16, 64)
