"""GPU parity of the next-token cross-entropy (gfn_cross_entropy_forward /
_backward through manifold_b200.losses) against torch's fp32
nn.CrossEntropyLoss on the same CUDA logits: the loss the reference's
training loops apply to logits.view(-1, V).

Tolerances (float32 arithmetic in both, different summation orders and
exponential implementations): loss |a - b| <= 1e-5 |b| + 1e-6; logit
gradients |a - b| <= 1e-5 max|b| + 1e-9.
"""
import pytest
import torch

import manifold_b200 as gfn
from manifold_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _pair(rows, V, scale=3.0, ignore_index=-100, n_ignored=0, seed=0, upstream=1.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, V, generator=g) * scale).to(DEV)
    t = torch.randint(0, V, (rows,), generator=g)
    if n_ignored:
        t[torch.randperm(rows, generator=g)[:n_ignored]] = ignore_index
    t = t.to(DEV)
    xa = x.clone().requires_grad_(True)
    la = gfn.CrossEntropyLoss(ignore_index=ignore_index)(xa, t)
    (la * upstream).backward()
    xb = x.clone().requires_grad_(True)
    lb = torch.nn.CrossEntropyLoss(ignore_index=ignore_index)(xb, t)
    (lb * upstream).backward()
    return la.detach(), lb.detach(), xa.grad, xb.grad


def _check(la, lb, ga, gb):
    assert torch.isfinite(la)
    assert abs(la.item() - lb.item()) <= 1e-5 * abs(lb.item()) + 1e-6, (la.item(), lb.item())
    err = (ga - gb).abs().max().item()
    assert err <= 1e-5 * gb.abs().max().item() + 1e-9, err


@pytest.mark.parametrize("rows,V", [(1, 4), (37, 1000), (64, 32000), (5, 1003), (3, 50257)])
def test_cross_entropy_matches_torch(rows, V):
    _check(*_pair(rows, V, seed=rows + V))


def test_cross_entropy_ignore_index_and_upstream_gradient():
    _check(*_pair(96, 4096, ignore_index=0, n_ignored=17, seed=3, upstream=2.5))
    _check(*_pair(40, 999, ignore_index=-100, n_ignored=9, seed=4, upstream=-0.75))


def test_cross_entropy_large_logits():
    # magnitudes where a naive exp overflows: the row max must be subtracted
    _check(*_pair(16, 2048, scale=300.0, seed=5))


def test_cross_entropy_sequence_shape():
    # [B, L, V] logits against [B, L] targets, as the training loops pass them
    g = torch.Generator().manual_seed(6)
    x = torch.randn(4, 9, 512, generator=g).to(DEV)
    t = torch.randint(0, 512, (4, 9), generator=g).to(DEV)
    xa = x.clone().requires_grad_(True)
    la = gfn.cross_entropy(xa, t)
    la.backward()
    xb = x.clone().requires_grad_(True)
    lb = torch.nn.functional.cross_entropy(xb.view(-1, 512), t.view(-1))
    lb.backward()
    _check(la.detach(), lb.detach(), xa.grad, xb.grad)


def test_cross_entropy_all_ignored_is_nan_like_torch():
    x = torch.randn(4, 64, device=DEV)
    t = torch.full((4,), -100, device=DEV, dtype=torch.int64)
    assert torch.isnan(gfn.cross_entropy(x, t))
    assert torch.isnan(torch.nn.functional.cross_entropy(x, t))


def test_cross_entropy_bad_target_flags_device_error():
    _lib.device_error(reset=True)
    x = torch.randn(3, 16, device=DEV)
    t = torch.tensor([1, 16, 2], device=DEV)  # 16 is outside [0, 16)
    loss = gfn.cross_entropy(x, t)
    assert torch.isnan(loss)
    assert _lib.device_error(reset=True) & 2


def test_cross_entropy_backward_in_place_over_logits():
    # the C ABI allows grad_logits == logits
    g = torch.Generator().manual_seed(7)
    x = torch.randn(8, 256, generator=g).to(DEV)
    t = torch.randint(0, 256, (8,), generator=g).to(DEV)
    rl = torch.empty(8, device=DEV)
    lse = torch.empty(8, 2, device=DEV)
    s = _lib.stream_of(x.device)
    _lib.call("gfn_cross_entropy_forward", _lib.ptr(x), _lib.ptr(t), 8, 256, -100, _lib.ptr(rl), _lib.ptr(lse), s)
    scale = torch.full((1,), 1.0 / 8, device=DEV)
    ref = torch.softmax(x, -1) / 8
    ref[torch.arange(8), t] -= 1.0 / 8
    _lib.call("gfn_cross_entropy_backward", _lib.ptr(x), _lib.ptr(t), _lib.ptr(lse), 8, 256, -100,
              _lib.ptr(scale), _lib.ptr(x), s)
    assert (x - ref).abs().max().item() <= 1e-7
