"""Per-module cache of quantised weights / weight scales, as coat/utils/_fp8_weightcache.py:5-43.

`prepare_weight(weight, name, is_first_microbatch)`:
  * first micro-batch: quantise the bf16 weight per tensor (one fused amax pass + one division /
    transpose pass on the GPU) and remember the result under `<name>_fp8`, `<name>_fp8_t`,
    `<name>_fp8_scale`;
  * later micro-batches: return what was remembered.
With `qargs.weight_memory_efficient` only the scale is kept (and returned); the autograd blocks then
re-derive the codes from the bf16 weight with `fp8_division[_transpose]` where they need them.
"""
import torch.nn as nn

from ..activation.real_quantization import fp8_division_transpose


class FP8CacheWeightModule(nn.Module):
    def __init__(self, config, qargs, layer_id):
        super().__init__()
        self.config = config
        self.qargs = qargs
        self.layer_id = layer_id

    def prepare_weight(self, weight, weight_name, is_first_microbatch):
        efficient = self.qargs.weight_memory_efficient
        if is_first_microbatch:
            w_fp8, w_s, w_fp8_t = fp8_division_transpose(weight, self.qargs.group_size, self.fwobits["fwbit"])
            setattr(self, f"{weight_name}_fp8_scale", w_s)
            if efficient:
                return w_s
            setattr(self, f"{weight_name}_fp8", w_fp8)
            setattr(self, f"{weight_name}_fp8_t", w_fp8_t)
            return w_fp8, w_fp8_t, w_s
        if efficient:
            return getattr(self, f"{weight_name}_fp8_scale")
        return (getattr(self, f"{weight_name}_fp8"), getattr(self, f"{weight_name}_fp8_t"),
                getattr(self, f"{weight_name}_fp8_scale"))

    def forward(self, x):
        pass
