"""Next-token cross-entropy on the library's kernels: the loss of the
reference's training loops, nn.CrossEntropyLoss() applied to
logits.view(-1, V) (demos/wikitext/train_wikitext.py:162,185; ignore_index
as in demos/copy_task/train_copy_task.py:175).

The forward reads the fp32 logits once (per-row max, log-sum-exp and loss,
gfn_cross_entropy_forward); the backward reads them once more and writes
d loss / d logits (gfn_cross_entropy_backward), with the upstream gradient
and 1 / (rows not ignored) as a device scalar.  Mean reduction and
ignore_index as torch's; class weights and label smoothing are not
implemented and raise GfnError.  CUDA tensors only.
"""
import torch
import torch.nn as nn

from . import _lib
from ._lib import GfnError, call, ptr, require_cuda


class CrossEntropyFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, ignore_index):
        V = logits.shape[-1]
        x = logits.reshape(-1, V)
        if x.dtype != torch.float32:
            raise GfnError("cross_entropy: logits must be float32")
        x = x.contiguous()
        t = target.reshape(-1).to(torch.int64).contiguous()
        if t.shape[0] != x.shape[0]:
            raise GfnError(f"cross_entropy: {x.shape[0]} logit rows but {t.shape[0]} targets")
        rows = x.shape[0]
        row_loss = torch.empty(rows, device=x.device, dtype=torch.float32)
        row_stats = torch.empty(rows, 2, device=x.device, dtype=torch.float32)  # (max, log sum exp)
        call("gfn_cross_entropy_forward", ptr(x), ptr(t), rows, V, int(ignore_index), ptr(row_loss),
             ptr(row_stats), _lib.stream_of(x.device))
        count = (t != ignore_index).sum().to(torch.float32)
        ctx.save_for_backward(x, t, row_stats, count)
        ctx.ignore_index = int(ignore_index)
        ctx.shape = logits.shape
        return row_loss.sum() / count

    @staticmethod
    def backward(ctx, g):
        x, t, row_stats, count = ctx.saved_tensors
        grad = torch.empty_like(x)
        scale = (g.to(torch.float32) / count).reshape(1).contiguous()
        call("gfn_cross_entropy_backward", ptr(x), ptr(t), ptr(row_stats), x.shape[0], x.shape[1],
             ctx.ignore_index, ptr(scale), ptr(grad), _lib.stream_of(x.device))
        return grad.reshape(ctx.shape), None, None


def cross_entropy(logits, target, ignore_index=-100):
    """Mean cross-entropy of logits [N, V] (or [..., V]) against targets [N]."""
    require_cuda(logits, target)
    return CrossEntropyFn.apply(logits, target, ignore_index)


class CrossEntropyLoss(nn.Module):
    """nn.CrossEntropyLoss(ignore_index=..., reduction="mean") on the kernels."""

    def __init__(self, weight=None, ignore_index=-100, reduction="mean", label_smoothing=0.0):
        super().__init__()
        if weight is not None or label_smoothing != 0.0 or reduction != "mean":
            raise GfnError("CrossEntropyLoss: only reduction='mean' without class weights or "
                           "label smoothing is implemented")
        self.ignore_index = ignore_index

    def forward(self, logits, target):
        return cross_entropy(logits, target, self.ignore_index)
