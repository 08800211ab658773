"""Cross-entropy loss head with the names and call signatures of the reference's
coat/activation/liger/cross_entropy.py (`LigerCrossEntropyFunction` :305-384, `liger_fixed_cross_entropy` :387-393,
`LigerForCausalLMLoss` :396-410), on one hand-written CUDA kernel (csrc/cross_entropy.cu) instead of the Triton
kernel: the loss of every row and, in place of the logits, its gradient, so that no second [tokens, vocabulary]
tensor exists.  Supported: what COAT's models use, i.e. hard labels with `ignore_index`, reduction "mean" / "sum" /
"none"; label smoothing, the z-loss term and soft-capping (options of the reference's kernel that its models never
switch on) raise.
"""
from typing import Optional

import torch

from ... import _lib


def cross_entropy_forward(_input, target, ignore_index, lse_square_scale, label_smoothing, reduction, softcap,
                          return_z_loss):
    """-> (loss, z_loss, _input) with `_input` overwritten by d loss / d _input (cross_entropy.py:212-278)."""
    if lse_square_scale != 0.0 or label_smoothing != 0.0 or softcap is not None or return_z_loss:
        raise NotImplementedError("coat_b200 cross entropy: label smoothing, z-loss and soft-capping are not provided")
    if reduction not in ("mean", "sum", "none"):
        raise ValueError(f"reduction {reduction!r}")
    if not _input.is_cuda:
        raise RuntimeError("coat_b200: the cross-entropy kernel needs CUDA tensors (no CPU path exists)")
    if _input.dim() != 2 or _input.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError("expected fp32 or bf16 logits of shape (tokens, vocabulary)")
    if _input.stride(-1) != 1:
        _input = _input.contiguous()
    target = target.contiguous().to(torch.int64)
    rows, V = _input.shape
    loss_1d = torch.empty(rows, dtype=torch.float32, device=_input.device)
    # the mean is over the rows that count; decided on the device, read once (the reference reads it the same way)
    n_non_ignore = int((target != ignore_index).sum().item()) if reduction == "mean" else 1
    inv_n = 1.0 / n_non_ignore if n_non_ignore > 0 else 0.0
    with torch.cuda.device(_input.device):
        _lib.check(_lib.lib().coat_cross_entropy_inplace(
            _input.data_ptr(), _lib.float_dtype(_input), _input.stride(0), target.data_ptr(), loss_1d.data_ptr(), rows, V,
            int(ignore_index), float(inv_n), _lib.stream_ptr(_input.device)), "cross_entropy_inplace")
    loss = loss_1d.to(_input.dtype) if reduction == "none" else loss_1d.sum().to(_input.dtype)
    return loss, None, _input


def cross_entropy_backward(_input, grad_output):
    """The stored gradient times the incoming one (cross_entropy.py:281-302); nothing to do for a gradient of 1."""
    if grad_output.numel() == 1:
        if float(grad_output) != 1.0:
            _input.mul_(grad_output.to(_input.dtype))
    else:   # reduction "none": one factor per row
        _input.mul_(grad_output.to(_input.dtype).unsqueeze(-1))
    return _input


class LigerCrossEntropyFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, _input, target, ignore_index: int = -100, lse_square_scale: float = 0.0,
                label_smoothing: float = 0.0, reduction: str = "mean", softcap: Optional[float] = None,
                return_z_loss: bool = False):
        loss, z_loss, _input = cross_entropy_forward(_input, target, ignore_index, lse_square_scale, label_smoothing,
                                                     reduction, softcap, return_z_loss)
        ctx.save_for_backward(_input.detach())
        ctx.return_z_loss = return_z_loss
        return loss, z_loss

    @staticmethod
    def backward(ctx, grad_output, grad_ouput2):
        (_input,) = ctx.saved_tensors
        return (cross_entropy_backward(_input, grad_output), None, None, None, None, None, None, None)


def liger_fixed_cross_entropy(source, target, num_items_in_batch: int = None, ignore_index: int = -100, **kwargs):
    reduction = "sum" if num_items_in_batch is not None else "mean"
    loss, _ = LigerCrossEntropyFunction.apply(source, target, ignore_index, 0.0, 0.0, reduction)
    if reduction == "sum":
        loss = loss / num_items_in_batch
    return loss


def LigerForCausalLMLoss(logits, labels, vocab_size: int, num_items_in_batch: int = None, ignore_index: int = -100,
                         **kwargs):
    """Shifted next-token loss (cross_entropy.py:396-410): logits in fp32, tokens < n predict n."""
    logits = logits.float()
    shift_logits = logits[..., :-1, :].contiguous().view(-1, vocab_size)
    shift_labels = labels[..., 1:].contiguous().view(-1).to(shift_logits.device)
    return liger_fixed_cross_entropy(shift_logits, shift_labels, num_items_in_batch, ignore_index, **kwargs)
