"""GPU parity of the multi-scheme integrator kernel: the reference's other
integrators (Euler, Heun, RK4, Verlet, Yoshida, Forest-Ruth, Omelyan,
Dormand-Prince) and the toroidal topology, as whole models against the
reference's own outputs (tests/golden/<case>.npz) and as single-head
operators against the oracle.  All calls go through the C ABI.

Tolerances: free-running sequences rtol 1e-4 / atol 1e-5 per row (the bar of
the other sequence tests); one operator step at the per-step bar.
"""
import os

import numpy as np
import pytest
import torch

import manifold_b200 as gfn
from manifold_b200.cuda import ops
from oracle import gfn_oracle as O
from tests.golden import cases as C
from tests.parity import report, rowwise_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda:0"


def cu(a):
    return torch.as_tensor(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("name", C.VARIANT_CASES)
def test_variant_model_matches_reference(name):
    cfg = C.CASES[name]
    P = C.make_params(cfg)
    g = dict(np.load(os.path.join(GOLD, f"{name}.npz")))
    torch.manual_seed(0)
    m = gfn.Manifold(**C.model_kwargs(cfg)).to(DEV).eval()
    C.load_into_model(m, cfg, P)
    with torch.no_grad():
        x_seq, v_seq, (x, v), _ = m.recurrence(cu(g["ids"]))
        out = m(cu(g["ids"]))
    report(x_seq.cpu().numpy(), g["x_seq"], f"{name} x_seq")
    rowwise_close(x_seq.cpu().numpy(), g["x_seq"], 1e-4, 1e-5, f"{name} x_seq")
    rowwise_close(v_seq.cpu().numpy(), g["v_seq"], 1e-4, 1e-5, f"{name} v_seq")
    rowwise_close(x.cpu().numpy(), g["x_final"], 1e-4, 1e-5, f"{name} x_final")
    assert len(out) == 6 and out[0].shape[:2] == g["ids"].shape


SCHEMES = ["euler", "heun", "rk4", "verlet", "yoshida", "forest_ruth", "omelyan", "dormand_prince"]


@pytest.mark.parametrize("scheme", SCHEMES)
@pytest.mark.parametrize("topology,hd,rank", [(0, 64, 4), (0, 96, 16), (1, 32, 4)])
def test_integrator_op_vs_oracle(scheme, topology, hd, rank):
    rng = np.random.default_rng(len(scheme) * 7 + hd + topology)
    B, f = 45, np.float32
    x = (rng.uniform(0, 6, (B, hd)) if topology else rng.standard_normal((B, hd))).astype(f)
    v = (rng.standard_normal((B, hd)) * 2).astype(f)
    F = rng.standard_normal((B, hd)).astype(f)
    U = (rng.standard_normal((hd, rank)) * 0.3).astype(f)
    W = (rng.standard_normal((hd, rank)) * 0.3).astype(f)
    fin = 2 * hd if topology else hd
    Wf = (rng.standard_normal((hd, fin)) * 0.1).astype(f)
    bf = (rng.standard_normal(hd) * 0.3).astype(f)
    Wi = (rng.standard_normal((hd, hd)) * 0.1).astype(f)
    xo, vo = O.integrator_step("rk45" if scheme == "dormand_prince" else scheme, x, v, F,
                               None if topology else U, None if topology else W, Wf, bf, Wi, 0.1,
                               np.float32(0.9), 2, topology)
    fn = getattr(ops, f"{scheme}_fused")
    xn, vn = fn(cu(x), cu(v), cu(F), None if topology else cu(U), None if topology else cu(W), 0.1, 0.9, 2,
                topology=topology, Wf=cu(Wf), bf=cu(bf), Wi=cu(Wi))
    rowwise_close(xn.cpu().numpy(), xo, 1e-5, 1e-6, f"{scheme} x")
    rowwise_close(vn.cpu().numpy(), vo, 1e-5, 1e-6, f"{scheme} v")


def test_heun_integrator_module_and_all_heads_launch():
    """HeunIntegrator (the reference's default) through its module, and the
    all-heads launch equal to per-head launches."""
    rng = np.random.default_rng(9)
    B, H, hd, r = 33, 4, 32, 4
    f = np.float32
    x = rng.standard_normal((B, H * hd)).astype(f)
    v = rng.standard_normal((B, H * hd)).astype(f)
    F = rng.standard_normal((B, H * hd)).astype(f)
    U = (rng.standard_normal((H, hd, r)) * 0.3).astype(f)
    W = (rng.standard_normal((H, hd, r)) * 0.3).astype(f)
    Wf = (rng.standard_normal((H, hd, hd)) * 0.1).astype(f)
    bf = (rng.standard_normal((H, hd)) * 0.3).astype(f)
    Wi = (rng.standard_normal((H, hd, hd)) * 0.1).astype(f)
    sc = np.array([0.8, 0.9, 1.0, 1.1], f)
    xa, va = ops.integrator_heads("heun", cu(x), cu(v), cu(F), cu(U), cu(W), 0.1, cu(sc), 1, 0, cu(Wf),
                                  cu(bf), cu(Wi), H)
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        ch = gfn.LowRankChristoffel(hd, r).to(DEV)
        with torch.no_grad():
            ch.U.copy_(cu(U[h])); ch.W.copy_(cu(W[h]))
            ch.forget_gate.weight.copy_(cu(Wf[h])); ch.forget_gate.bias.copy_(cu(bf[h]))
            ch.input_gate.weight.copy_(cu(Wi[h]))
            xh, vh = gfn.HeunIntegrator(ch, dt=0.1)(cu(x[:, sl]), cu(v[:, sl]), force=cu(F[:, sl]),
                                                    dt_scale=float(sc[h]))
        np.testing.assert_array_equal(xh.cpu().numpy(), xa[:, sl].cpu().numpy())
        np.testing.assert_array_equal(vh.cpu().numpy(), va[:, sl].cpu().numpy())
