"""`CoatFP8Trainer`: a transformers `Trainer` whose optimizer is the FP8 `CoatAdamW`
(coat/fp8_trainer.py:130-170).  Parameters named by `Trainer.get_decay_parameter_names` get the configured
weight decay, the rest none; lr / betas / eps come from the training arguments and `coat_args` (a
`QuantizationConfig`) selects the optimizer-state formats.

transformers is imported only when the class is first asked for, so that the rest of the package does not
depend on it; `coat_optimizer_groups` and `build_coat_optimizer` hold the logic and work without it.
"""
import os

import torch

from .optimizer.fp8_adamw import CoatAdamW


def get_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK") or 0)


def coat_optimizer_groups(named_parameters, decay_parameter_names, weight_decay):
    """Two parameter groups: trainable parameters that decay, and those that do not."""
    named = [(n, p) for n, p in named_parameters if p.requires_grad]
    decay = set(decay_parameter_names)
    return [
        {"params": [p for n, p in named if n in decay], "weight_decay": weight_decay},
        {"params": [p for n, p in named if n not in decay], "weight_decay": 0.0},
    ]


def build_coat_optimizer(model, args, decay_parameter_names, qargs=None):
    """args: anything with learning_rate, adam_beta1, adam_beta2, adam_epsilon, weight_decay
    (transformers.TrainingArguments has them)."""
    groups = coat_optimizer_groups(model.named_parameters(), decay_parameter_names, args.weight_decay)
    kwargs = {"lr": args.learning_rate, "betas": (args.adam_beta1, args.adam_beta2), "eps": args.adam_epsilon}
    if qargs is not None:
        kwargs["qargs"] = qargs
    return CoatAdamW(groups, **kwargs)


class MasterWeights:
    """fp32 master copies of a bf16 model's parameters.  CoatAdamW steps fp32 parameters (like the reference's
    kernel, whose per-group vectors are float32 by contract) while the FP8 layers compute on bf16 weights; in
    the reference the surrounding framework (DeepSpeed / FSDP mixed precision) holds the masters.  This is
    the single-process form: the optimizer is built over `named_parameters()` of this object, `copy_grads()`
    hands it the model's gradients in fp32, and after `attach(optimizer)` every step writes the bf16 model
    weights from inside the optimizer kernel."""

    def __init__(self, model):
        self.names, self.model_params, self.masters = [], [], []
        for name, p in model.named_parameters():
            if not p.requires_grad:
                continue
            self.names.append(name)
            self.model_params.append(p)
            self.masters.append(torch.nn.Parameter(p.detach().float().clone()))

    def named_parameters(self):
        return list(zip(self.names, self.masters))

    def attach(self, optimizer):
        optimizer.attach_bf16_weights(
            (m, p.data) for m, p in zip(self.masters, self.model_params) if p.dtype == torch.bfloat16)

    @torch.no_grad()
    def copy_grads(self, zero_model_grads=True):
        for m, p in zip(self.masters, self.model_params):
            if p.grad is None:
                m.grad = None
                continue
            if m.grad is None:
                m.grad = p.grad.float()
            else:
                m.grad.copy_(p.grad)
            if zero_model_grads:
                p.grad = None

    @torch.no_grad()
    def write_back(self):
        """For parameters that are not bf16 (no fused copy): master -> model."""
        for m, p in zip(self.masters, self.model_params):
            if p.dtype != torch.bfloat16:
                p.copy_(m)


_trainer_class = None


def _make_trainer_class():
    from transformers import Trainer

    class CoatFP8Trainer(Trainer):
        def __init__(self, coat_args=None, *args, **kwargs):
            super().__init__(*args, **kwargs)
            self.qargs = coat_args

        def create_optimizer(self):
            if get_local_rank() == 0:
                print("Setup the COAT FP8 optimizer")
            if self.optimizer is None:
                self.optimizer = build_coat_optimizer(self.model, self.args,
                                                      self.get_decay_parameter_names(self.model), self.qargs)
            return self.optimizer

    return CoatFP8Trainer


def __getattr__(name):
    global _trainer_class
    if name == "CoatFP8Trainer":
        if _trainer_class is None:
            _trainer_class = _make_trainer_class()
        return _trainer_class
    raise AttributeError(name)
