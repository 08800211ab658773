"""Global FP8 state, as coat/utils/_fp8manager.py:20-25: the training loop sets `is_first_microbatch`
to True for the first micro-batch after an optimizer step (weights changed: their per-tensor scales
are recomputed and cached) and to False for the others (cached scales are reused)."""


class FP8Manager:
    is_first_microbatch = True
