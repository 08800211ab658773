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
