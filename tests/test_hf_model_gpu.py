"""A stock transformers Llama checkpoint through the whole path on the GPU: `download_and_convert_llama` ->
`AutoModelForCausalLM.from_pretrained` (the registered COAT classes) -> training mode in bf16 with the FP8 activation
stream and FP8 linears -> FP8 optimizer steps on fp32 masters (the route of the reference's ToolBench example:
convert, load, `CoatFP8Trainer.create_optimizer`, train).  Checked: the FP8 training loss is within 2 % of the stock
model's loss on the same tokens (FP8 tolerance, as in test_llama_model_gpu.py), and ten steps reduce it."""
from types import SimpleNamespace

import pytest
import torch

transformers = pytest.importorskip("transformers")
pytestmark = pytest.mark.gpu


def test_converted_stock_checkpoint_trains(tmp_path):
    from transformers import AutoModelForCausalLM, LlamaConfig, LlamaForCausalLM

    from coat_b200.fp8_trainer import MasterWeights, build_coat_optimizer
    from coat_b200.models.hf import CoatLlamaForCausalLM, ConvertArguments, download_and_convert_llama
    from coat_b200.utils._fp8_quantization_config import QuantizationConfig
    from coat_b200.utils._fp8manager import FP8Manager
    cfg = LlamaConfig(hidden_size=256, intermediate_size=768, num_attention_heads=4, num_key_value_heads=4,
                      num_hidden_layers=2, vocab_size=512, max_position_embeddings=256, rms_norm_eps=1e-5)
    torch.manual_seed(5)
    stock = LlamaForCausalLM(cfg)
    stock.save_pretrained(tmp_path / "stock")
    download_and_convert_llama(ConvertArguments(str(tmp_path / "stock"), str(tmp_path / "coat")),
                               QuantizationConfig(group_size=16, weight_memory_efficient=True))
    model = AutoModelForCausalLM.from_pretrained(tmp_path / "coat", torch_dtype=torch.bfloat16).cuda()
    assert isinstance(model, CoatLlamaForCausalLM)
    ids = torch.randint(0, 512, (2, 128), generator=torch.Generator().manual_seed(6)).cuda()
    with torch.no_grad():
        want = float(stock.cuda().eval()(ids, labels=ids).loss)
    model.train()
    FP8Manager.is_first_microbatch = True
    first = float(model(input_ids=ids, labels=ids).loss.detach())
    assert abs(first - want) <= 0.02 * want, (first, want)

    args = SimpleNamespace(learning_rate=2e-3, adam_beta1=0.9, adam_beta2=0.95, adam_epsilon=1e-8, weight_decay=0.0)
    masters = MasterWeights(model)
    opt = build_coat_optimizer(masters, args, [n for n, p in model.named_parameters() if p.dim() == 2])
    masters.attach(opt)
    losses = []
    for _ in range(10):
        FP8Manager.is_first_microbatch = True
        loss = model(input_ids=ids, labels=ids).loss
        loss.backward()
        masters.copy_grads()
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < 0.8 * losses[0], losses
