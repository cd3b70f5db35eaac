"""GPU parity of the single-head operators of the gfn.cuda boundary:
forward and backward of the low-rank and toroidal Christoffel terms and of
the leapfrog integrator (input gate, forget stacks, torus), against the
reference's own outputs and autograd gradients (tests/golden/ops.npz) and
the oracle; recurrent_manifold_fused against the oracle.  All calls go
through the C ABI.

Tolerances: forward values at the per-step bar (|a - b| <= 1e-6 + 1e-5 max|b_row|);
gradients |a - b| <= 1e-5 + 2e-3 max|b| (the bar of the other gradient tests).
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


def G():
    return dict(np.load(os.path.join(GOLD, "ops.npz")))


def cu(a, grad=False):
    t = torch.as_tensor(np.ascontiguousarray(a)).to(DEV)
    return t.requires_grad_(True) if grad else t


def grad_close(a, b, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    tol = 1e-5 + 2e-3 * np.max(np.abs(b))
    err = np.max(np.abs(a - b))
    assert err <= tol, f"{what}: max err {err:.3e} > {tol:.3e}"


def test_christoffel_backward_matches_reference():
    g = G()
    v, U, W = cu(g["lr_v"], True), cu(g["lr_U"], True), cu(g["lr_W"], True)
    gam = ops.christoffel_fused(v, U, W)
    rowwise_close(gam.detach().cpu().numpy(), g["lr_gamma"], what="gamma")
    (gam * cu(g["lr_G"])).sum().backward()
    grad_close(v.grad.cpu(), g["lr_dv"], "dv")
    grad_close(U.grad.cpu(), g["lr_dU"], "dU")
    grad_close(W.grad.cpu(), g["lr_dW"], "dW")
    # the binding-level entry returns the reference's 5-list
    out = ops.christoffel_backward(cu(g["lr_G"]), cu(g["lr_v"]), cu(g["lr_U"]), cu(g["lr_W"]))
    assert len(out) == 5 and out[3] is None and out[4] is None
    grad_close(out[0].cpu(), g["lr_dv"], "dv (binding)")


def test_torus_christoffel_forward_backward_matches_reference():
    g = G()
    v, x = cu(g["lr_v"], True), cu(g["tor_x"], True)
    tc = gfn.ToroidalChristoffel(v.shape[1]).to(DEV)
    tc.return_friction_separately = True
    gam, _ = tc(v, x)
    rowwise_close(gam.detach().cpu().numpy(), g["tor_gamma"], what="torus gamma")
    (gam * cu(g["lr_G"])).sum().backward()
    grad_close(v.grad.cpu(), g["tor_dv"], "torus dv")
    grad_close(x.grad.cpu(), g["tor_dx"], "torus dx")


def _lowrank(g):
    hd, r = g["lr_U"].shape
    ch = gfn.LowRankChristoffel(hd, r).to(DEV)
    with torch.no_grad():
        ch.U.copy_(cu(g["lr_U"]))
        ch.W.copy_(cu(g["lr_W"]))
    return ch


def test_leapfrog_input_gate_forward_backward_matches_reference():
    """LeapfrogIntegrator without forget stacks: friction from the
    Christoffel's own gates, 5 sigmoid(forget_gate(x) + input_gate(F))."""
    g = G()
    ch = _lowrank(g)
    with torch.no_grad():
        ch.forget_gate.weight.copy_(cu(g["ig_Wf"]))
        ch.forget_gate.bias.copy_(cu(g["ig_bf"]))
        ch.input_gate.weight.copy_(cu(g["ig_Wi"]))
    integ = gfn.LeapfrogIntegrator(ch, dt=0.1)
    x, v, F = cu(g["ig_x"], True), cu(g["lr_v"], True), cu(g["ig_F"], True)
    xn, vn = integ(x, v, force=F, dt_scale=torch.tensor(0.87, device=DEV), steps=2)
    report(vn.detach().cpu().numpy(), g["ig_vn"], "input-gate leapfrog v")
    rowwise_close(xn.detach().cpu().numpy(), g["ig_xn"], what="x")
    rowwise_close(vn.detach().cpu().numpy(), g["ig_vn"], what="v")
    ((xn * cu(g["ig_Gx"])).sum() + (vn * cu(g["ig_Gv"])).sum()).backward()
    for nm, a in [("dx", x.grad), ("dv", v.grad), ("dF", F.grad), ("dU", ch.U.grad), ("dW", ch.W.grad),
                  ("dWf", ch.forget_gate.weight.grad), ("dbf", ch.forget_gate.bias.grad),
                  ("dWi", ch.input_gate.weight.grad)]:
        grad_close(a.cpu(), g["ig_" + nm], "input gate " + nm)


def test_leapfrog_forget_stack_backward_matches_reference():
    g = G()
    ch = _lowrank(g)
    integ = gfn.LeapfrogIntegrator(ch, dt=0.1)
    x, v, F = cu(g["ig_x"], True), cu(g["lr_v"], True), cu(g["ig_F"], True)
    wf, bf = cu(g["ig_Wf"][None], True), cu(g["ig_bf"][None], True)
    xn, vn = integ(x, v, force=F, dt_scale=torch.tensor(1.13, device=DEV), steps=3,
                   W_forget_stack=wf, b_forget_stack=bf, topology=0)
    rowwise_close(xn.detach().cpu().numpy(), g["st_xn"], what="x")
    rowwise_close(vn.detach().cpu().numpy(), g["st_vn"], what="v")
    ((xn * cu(g["ig_Gx"])).sum() + (vn * cu(g["ig_Gv"])).sum()).backward()
    for nm, a in [("dx", x.grad), ("dv", v.grad), ("dF", F.grad), ("dU", ch.U.grad), ("dW", ch.W.grad),
                  ("dWf", wf.grad[0]), ("dbf", bf.grad[0])]:
        grad_close(a.cpu(), g["st_" + nm], "forget stack " + nm)


def test_torus_leapfrog_forward_backward_matches_reference():
    g = G()
    hd = g["lr_v"].shape[1]
    tc = gfn.ToroidalChristoffel(hd, physics_config={"topology": {"type": "torus"}}).to(DEV)
    integ = gfn.LeapfrogIntegrator(tc, dt=0.1)
    x, v, F = cu(g["tor_x"], True), cu(g["lr_v"], True), cu(g["ig_F"], True)
    wf, bf = cu(g["tl_Wf"][None], True), cu(g["ig_bf"][None], True)
    xn, vn = integ(x, v, force=F, dt_scale=torch.tensor(0.95, device=DEV), steps=2,
                   W_forget_stack=wf, b_forget_stack=bf, topology=1)
    rowwise_close(xn.detach().cpu().numpy(), g["tl_xn"], what="torus x")
    rowwise_close(vn.detach().cpu().numpy(), g["tl_vn"], what="torus v")
    ((xn * cu(g["ig_Gx"])).sum() + (vn * cu(g["ig_Gv"])).sum()).backward()
    for nm, a in [("dx", x.grad), ("dv", v.grad), ("dF", F.grad), ("dWf", wf.grad[0]), ("dbf", bf.grad[0])]:
        grad_close(a.cpu(), g["tl_" + nm], "torus " + nm)


@pytest.mark.parametrize("hd,rank,B,topology", [(16, 4, 1, 0), (64, 16, 37, 0), (128, 8, 300, 0),
                                                (160, 4, 5, 0), (48, 4, 70, 1), (128, 4, 9, 1)])
def test_gated_leapfrog_shapes_vs_oracle(hd, rank, B, topology):
    rng = np.random.default_rng(hd + rank + B)
    f = np.float32
    x = (rng.uniform(0, 6, (B, hd)) if topology else rng.standard_normal((B, hd))).astype(f)
    v = (rng.standard_normal((B, hd)) * 2).astype(f)
    F = rng.standard_normal((B, hd)).astype(f)
    U = (rng.standard_normal((hd, rank)) * 0.3).astype(f)
    W = (rng.standard_normal((hd, rank)) * 0.3).astype(f)
    fin = 2 * hd if topology else hd
    Wf = (rng.standard_normal((hd, fin)) * 0.1).astype(f)
    bf = (rng.standard_normal(hd) * 0.3).astype(f)
    Wi = (rng.standard_normal((hd, hd)) * 0.1).astype(f)
    scale = rng.uniform(0.5, 1.5, B).astype(f)
    xo, vo = O.leapfrog_head_step_gated(x, v, F, None if topology else U, None if topology else W, Wf, bf,
                                        Wi, 0.1, scale[:, None], 2, topology)
    xn, vn = ops.leapfrog_fused(cu(x), cu(v), cu(F), None if topology else cu(U),
                                None if topology else cu(W), 0.1, cu(scale), 2, topology=topology,
                                Wf=cu(Wf), bf=cu(bf), Wi=cu(Wi))
    rowwise_close(xn.cpu().numpy(), xo, what="x")
    rowwise_close(vn.cpu().numpy(), vo, what="v")


def test_leapfrog_backward_vs_float64_autograd_many_steps():
    """A longer replay (5 steps, 128 rows, head_dim 64, rank 16) against
    float64 autograd of a torch restatement of the same step."""
    rng = np.random.default_rng(5)
    B, hd, r, steps = 128, 64, 16, 5
    f = np.float32
    arrs = dict(x=rng.standard_normal((B, hd)), v=rng.standard_normal((B, hd)) * 2,
                F=rng.standard_normal((B, hd)), U=rng.standard_normal((hd, r)) * 0.2,
                W=rng.standard_normal((hd, r)) * 0.2, Wf=rng.standard_normal((hd, hd)) * 0.1,
                bf=rng.standard_normal(hd) * 0.3, Wi=rng.standard_normal((hd, hd)) * 0.1)
    arrs = {k: a.astype(f) for k, a in arrs.items()}
    Gx, Gv = rng.standard_normal((B, hd)), rng.standard_normal((B, hd))

    def step64(t):
        x, v, F, U, W, Wf, bf, Wi = (t[k] for k in ("x", "v", "F", "U", "W", "Wf", "bf", "Wi"))
        eff = 0.1 * 0.9
        h = 0.5 * eff

        def gam(vv):
            p = vv @ U
            s = 1.0 / (1.0 + p.norm(dim=-1, keepdim=True) + 1e-6)
            return 20 * torch.tanh(((p * p) * s) @ W.T / 20)

        def mu(xx):
            return torch.sigmoid(xx @ Wf.T + bf + F @ Wi.T) * 5

        for _ in range(steps):
            vh = (v + h * (F - gam(v))) / (1 + h * mu(x))
            x = x + eff * vh
            v = (vh + h * (F - gam(vh))) / (1 + h * mu(x))
        return x, v

    t64 = {k: torch.tensor(a, dtype=torch.float64, requires_grad=True) for k, a in arrs.items()}
    x64, v64 = step64(t64)
    ((x64 * torch.tensor(Gx)).sum() + (v64 * torch.tensor(Gv)).sum()).backward()
    tg = {k: cu(a, True) for k, a in arrs.items()}
    xn, vn = ops.leapfrog_fused(tg["x"], tg["v"], tg["F"], tg["U"], tg["W"], 0.1, 0.9, steps,
                                Wf=tg["Wf"], bf=tg["bf"], Wi=tg["Wi"])
    ((xn * cu(Gx.astype(f))).sum() + (vn * cu(Gv.astype(f))).sum()).backward()
    for k in arrs:
        grad_close(tg[k].grad.cpu(), t64[k].grad.detach().numpy(), "d" + k)


def test_christoffel_backward_shapes_vs_float64():
    for hd, r, B in [(16, 4, 3), (96, 8, 257), (256, 16, 64)]:
        rng = np.random.default_rng(hd * r)
        v = torch.tensor(rng.standard_normal((B, hd)) * 3, dtype=torch.float64, requires_grad=True)
        U = torch.tensor(rng.standard_normal((hd, r)) * 0.3, dtype=torch.float64, requires_grad=True)
        W = torch.tensor(rng.standard_normal((hd, r)) * 0.3, dtype=torch.float64, requires_grad=True)
        Gm = torch.tensor(rng.standard_normal((B, hd)))
        p = v @ U
        s = 1.0 / (1.0 + p.norm(dim=-1, keepdim=True) + 1e-6)
        (20 * torch.tanh(((p * p) * s) @ W.T / 20) * Gm).sum().backward()
        out = ops.christoffel_backward(cu(Gm.float().numpy()), cu(v.detach().float().numpy()),
                                       cu(U.detach().float().numpy()), cu(W.detach().float().numpy()))
        grad_close(out[0].cpu(), v.grad.numpy(), f"dv {hd}/{r}")
        grad_close(out[1].cpu(), U.grad.numpy(), f"dU {hd}/{r}")
        grad_close(out[2].cpu(), W.grad.numpy(), f"dW {hd}/{r}")


def test_reactive_christoffel_is_the_plain_term_without_active_inference():
    g = G()
    a = ops.reactive_christoffel(cu(g["lr_v"]), cu(g["lr_U"]), cu(g["lr_W"]))
    rowwise_close(a.cpu().numpy(), g["lr_gamma"], what="reactive gamma")
    with pytest.raises(gfn.GfnError):
        ops.reactive_christoffel(cu(g["lr_v"]), cu(g["lr_U"]), cu(g["lr_W"]), plasticity=0.1)


def test_recurrent_manifold_fused_matches_oracle():
    """The reference-signature whole-sequence entry: stacked operands, one
    mixing matrix for every layer, dt scales of the first layer."""
    cfg = dict(C.CASES["c1"], B=6, L=5)
    P = C.make_params(cfg)
    d, H, NL = cfg["d"], cfg["H"], cfg["NL"]
    hd = d // H
    L0 = P["layers"][0]
    layers = []
    for lp in P["layers"]:
        q = dict(lp)
        q.update(Wx=L0["Wx"], Wv=L0["Wv"], bx=np.zeros(d, np.float32), bv=np.zeros(d, np.float32),
                 gx=np.ones(d, np.float32), gv=np.ones(d, np.float32), dt_params=L0["dt_params"])
        layers.append(q)
    rng = np.random.default_rng(3)
    F = rng.standard_normal((cfg["B"], cfg["L"], d)).astype(np.float32)
    x0 = rng.standard_normal((cfg["B"], d)).astype(np.float32)
    v0 = rng.standard_normal((cfg["B"], d)).astype(np.float32)
    xs, _, xf, vf = O.manifold_forward(x0, v0, F, layers, H, cfg["dt"])
    def st(k):
        return cu(np.concatenate([lp[k] for lp in P["layers"]], 0))

    dt_scales = O.softplus(L0["dt_params"])
    out = ops.recurrent_manifold_fused(cu(x0), cu(v0), cu(F), st("U"), st("W"), cfg["dt"], cu(dt_scales),
                                       None, H, mix_x=cu(L0["Wx"]), mix_v=cu(L0["Wv"]), Wf=st("Wf"),
                                       Wi=st("Wi"), bf=st("bf"))
    x_final, v_final, x_seq, reg = out
    rowwise_close(x_seq.cpu().numpy(), xs, 1e-4, 1e-5, "x_seq")
    rowwise_close(x_final.cpu().numpy(), xf, 1e-4, 1e-5, "x_final")
    rowwise_close(v_final.cpu().numpy(), vf, 1e-4, 1e-5, "v_final")
    assert float(reg) == 0.0

