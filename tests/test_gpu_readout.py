"""Readout GEMMs through the split-fp16 tensor-core path vs float64.

The readout nn.Linear(d -> vocab) runs as fp16 GEMMs over operands split into
two fp16 pieces (manifold_b200.readout).  Each product keeps ~22 bits, so
the result carries a few float32 ulps more error than a plain float32 GEMM
(measured ~1.4e-6 relative for the logits vs 2.9e-7).  Bar, for the logits
and both gradients: relative L2 error against float64 at most
max(8 x torch's float32 GEMM error, 3e-6); rows span several chunks.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.double() - b).norm() / b.norm()).item()


def test_split_readout_matches_float64(monkeypatch):
    from manifold_b200 import readout as R
    monkeypatch.setattr(R, "CHUNK_ROWS", 1024)
    torch.manual_seed(0)
    M, d, V = 2500, 256, 1000
    lin = torch.nn.Linear(d, V).cuda()
    y = torch.randn(M, d, device="cuda") * 3
    g = torch.randn(M, V, device="cuda") * 1e-5  # the size of a mean CE gradient

    y1 = y.clone().requires_grad_(True)
    out = R.readout_linear(y1, lin)
    out.backward(g)
    dy, dW, db = y1.grad, lin.weight.grad.clone(), lin.bias.grad.clone()
    lin.weight.grad = None
    lin.bias.grad = None

    y2 = y.clone().requires_grad_(True)  # torch fp32 for the error scale
    out32 = torch.nn.functional.linear(y2, lin.weight, lin.bias)
    out32.backward(g)

    yd, Wd, bd, gd = y.double(), lin.weight.double(), lin.bias.double(), g.double()
    ref = yd @ Wd.T + bd
    for name, a, a32, b in (("logits", out, out32, ref), ("dy", dy, y2.grad, gd @ Wd),
                            ("dW", dW, lin.weight.grad, gd.T @ yd), ("db", db, lin.bias.grad, gd.sum(0))):
        e, e32 = _rel(a, b), _rel(a32, b)
        assert e <= max(8 * e32, 3e-6), (name, e, e32)


def test_model_readout_uses_split_path():
    import manifold_b200 as gfn
    torch.manual_seed(0)
    m = gfn.Manifold(vocab_size=300, dim=64, depth=1, rank=16, heads=2,
                     integrator_type="leapfrog").cuda().eval()
    ids = torch.randint(0, 300, (4, 5), device="cuda")
    with torch.no_grad():
        a = m(ids)[0]
        m.readout_split = False
        b = m(ids)[0]
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
