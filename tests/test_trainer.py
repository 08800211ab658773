"""CPU tests of the trainer glue: parameter grouping and optimizer construction (no step: the step needs
the GPU library)."""
from types import SimpleNamespace

import torch

from coat_b200.fp8_trainer import build_coat_optimizer, coat_optimizer_groups
from coat_b200.utils._fp8_quantization_config import QuantizationConfig


class Tiny(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.proj = torch.nn.Linear(128, 256)
        self.norm = torch.nn.LayerNorm(256)
        self.frozen = torch.nn.Linear(8, 8)
        for p in self.frozen.parameters():
            p.requires_grad_(False)


def test_groups_split_decay_and_skip_frozen():
    m = Tiny()
    groups = coat_optimizer_groups(m.named_parameters(), ["proj.weight"], 0.1)
    assert [g["weight_decay"] for g in groups] == [0.1, 0.0]
    assert groups[0]["params"] == [m.proj.weight]
    assert {id(p) for p in groups[1]["params"]} == {id(m.proj.bias), id(m.norm.weight), id(m.norm.bias)}


def test_build_optimizer_takes_hyperparameters_from_args():
    m = Tiny()
    args = SimpleNamespace(learning_rate=3e-4, adam_beta1=0.9, adam_beta2=0.95, adam_epsilon=1e-6, weight_decay=0.05)
    opt = build_coat_optimizer(m, args, ["proj.weight"], QuantizationConfig())
    assert len(opt.param_groups) == 2
    for g, wd in zip(opt.param_groups, (0.05, 0.0)):
        assert g["lr"] == 3e-4 and g["betas"] == (0.9, 0.95) and g["eps"] == 1e-6 and g["weight_decay"] == wd
    assert opt.param_groups[0]["params"] == [m.proj.weight]


def test_trainer_class_is_a_transformers_trainer():
    import pytest
    transformers = pytest.importorskip("transformers")
    from coat_b200 import fp8_trainer
    cls = fp8_trainer.CoatFP8Trainer
    assert issubclass(cls, transformers.Trainer) and "create_optimizer" in cls.__dict__
