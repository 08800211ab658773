"""The loss head of the reference (coat/activation/liger/): cross entropy whose gradient overwrites the logits."""
from .cross_entropy import LigerCrossEntropyFunction, LigerForCausalLMLoss, liger_fixed_cross_entropy  # noqa: F401
