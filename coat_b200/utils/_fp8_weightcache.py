"""Per-module cache of quantised weights / weight scales (coat/utils/_fp8_weightcache.py:5-43).

`prepare_weight(weight, name, is_first_microbatch)` quantises a bf16 weight per tensor on the first
micro-batch after an optimizer step (one amax pass, and unless only the scale is kept one division / transpose
pass on the GPU) and
hands back what it remembered on the following ones.  What is remembered, as module attributes with the
reference's names: `<name>_fp8_scale` always, `<name>_fp8` and `<name>_fp8_t` unless
`qargs.weight_memory_efficient` (then only the scale is returned and the autograd blocks re-derive the
codes from the bf16 weight where they need them)."""
import torch.nn as nn

from ..activation.real_quantization import fp8_division_transpose
from ..activation.real_quantization._ops import fp8_pertensor_scale

_SUFFIXES = ("_fp8", "_fp8_t", "_fp8_scale")


class FP8CacheWeightModule(nn.Module):
    def __init__(self, config, qargs, layer_id):
        super().__init__()
        self.config, self.qargs, self.layer_id = config, qargs, layer_id

    def _recall(self, weight_name):
        return tuple(getattr(self, weight_name + suffix) for suffix in _SUFFIXES)

    def prepare_weight(self, weight, weight_name, is_first_microbatch):
        scale_only = self.qargs.weight_memory_efficient
        if is_first_microbatch:
            if scale_only:   # the codes would be thrown away: one amax pass gives the same scale
                kept = (None, None, fp8_pertensor_scale(weight, self.fwobits["fwbit"]))
            else:
                codes, scale, codes_t = fp8_division_transpose(weight, self.qargs.group_size, self.fwobits["fwbit"])
                kept = (codes, codes_t, scale)
            for suffix, value in zip(_SUFFIXES, kept):
                if value is not None:
                    setattr(self, weight_name + suffix, value)
        if scale_only:
            return getattr(self, weight_name + "_fp8_scale")
        return self._recall(weight_name)

    def forward(self, x):
        pass
