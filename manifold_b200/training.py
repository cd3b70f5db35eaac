"""Training (autograd) path of Manifold: placeholder until the BPTT kernels land."""
from ._lib import GfnError


def manifold_train_forward(model, input_ids, attention_mask, state, force_manual):
    raise GfnError("gradients through the fused recurrence are not built yet; run under "
                   "torch.no_grad() or set requires_grad_(False)")
