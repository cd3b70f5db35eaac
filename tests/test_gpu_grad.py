"""BPTT backward on the GPU vs the reference's autograd (golden fixtures) and
vs the numpy oracle's backward at C5 layer shapes.

Tolerance: max |a - b| <= 1e-5 + 2e-3 * max|b| per gradient tensor (float32
gradients accumulated over tokens x layers in a different order)."""
import os

import numpy as np
import pytest
import torch

from oracle import gfn_oracle as O
from tests.golden import cases as C

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
RTOL, ATOL = 2e-3, 1e-5


def gclose(a, b, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(float(np.max(np.abs(b))), 1e-30)
    err = float(np.max(np.abs(a - b)))
    assert err <= ATOL + RTOL * scale, f"{what}: max |diff| {err:.3e} vs scale {scale:.3e}"


def cu(a):
    return torch.as_tensor(np.asarray(a)).cuda()


def build(cfg, P):
    import manifold_b200 as gfn
    torch.manual_seed(0)
    m = gfn.Manifold(**C.model_kwargs(cfg)).cuda()
    C.load_into_model(m, cfg, P)
    return m


def run_grad(cfg, P, ids, Gx, Gv, gxf, gvf, mask=None):
    m = build(cfg, P)
    F = cu(P["emb"][ids]).requires_grad_(True)
    _, (x, v), _, v_seq, x_seq, _ = m(force_manual=F, attention_mask=None if mask is None else cu(mask))
    loss = (torch.stack(x_seq, 1) * cu(Gx)).sum() + (torch.stack(v_seq, 1) * cu(Gv)).sum() \
        + (x * cu(gxf)).sum() + (v * cu(gvf)).sum()
    loss.backward()
    return m, F


@pytest.mark.parametrize("name", list(C.GRAD_CASES))
def test_backward_matches_reference_autograd(name):
    cfg = C.GRAD_CASES[name]
    g = dict(np.load(os.path.join(GOLD, f"{name}.npz")))
    P = C.make_params(cfg)
    m, F = run_grad(cfg, P, g["ids"], g["Gx"], g["Gv"], g["gxf"], g["gvf"], g.get("mask"))
    gclose(F.grad.cpu(), g["g_forces"], "forces")
    gclose(m.x0.grad.cpu()[0], g["g_x0"], "x0")
    gclose(m.v0.grad.cpu()[0], g["g_v0"], "v0")
    for l, layer in enumerate(m.layers):
        gclose(layer.dt_params.grad.cpu(), g[f"l{l}_dt_params"], f"l{l} dt_params")
        gclose(torch.stack([c.U.grad for c in layer.christoffels]).cpu(), g[f"l{l}_U"], f"l{l} U")
        gclose(torch.stack([c.W.grad for c in layer.christoffels]).cpu(), g[f"l{l}_W"], f"l{l} W")
        gclose(torch.stack([c.forget_gate.weight.grad for c in layer.christoffels]).cpu(),
               g[f"l{l}_Wf"], f"l{l} Wf")
        gclose(torch.stack([c.forget_gate.bias.grad for c in layer.christoffels]).cpu(),
               g[f"l{l}_bf"], f"l{l} bf")
        if cfg["H"] > 1:
            for nm in ("x", "v"):
                gW = getattr(layer, "out_proj_" + nm).weight.grad.cpu().numpy()
                if f"l{l}_W{nm}" in g:
                    gclose(gW, g[f"l{l}_W{nm}"], f"l{l} W{nm}")
                else:
                    gclose(gW.sum(1), g[f"l{l}_W{nm}_rowsum"], f"l{l} W{nm} rows")
                    gclose(gW.sum(0), g[f"l{l}_W{nm}_colsum"], f"l{l} W{nm} cols")
                    gclose(gW[:16, :16], g[f"l{l}_W{nm}_corner"], f"l{l} W{nm} corner")
                gclose(getattr(layer, "out_proj_" + nm).bias.grad.cpu(), g[f"l{l}_b{nm}"], f"l{l} b{nm}")
                gclose(getattr(layer, "mixed_norm_" + nm).weight.grad.cpu(), g[f"l{l}_g{nm}"],
                       f"l{l} g{nm}")


def test_backward_c5_shapes_vs_oracle_and_deterministic():
    """C5 layer shapes (d=512, 8 layers, 8 heads, r=4) at batch 64, 3 tokens."""
    cfg = dict(C.CASES["c5s"], B=64, L=3, seed=41, V=500)
    P = C.make_params(cfg)
    rng = np.random.default_rng(3)
    B, L, d = 64, 3, cfg["d"]
    ids = rng.integers(0, cfg["V"], (B, L))
    Gx = rng.standard_normal((B, L, d)).astype(np.float32)
    Gv = rng.standard_normal((B, L, d)).astype(np.float32)
    z = np.zeros((B, d), np.float32)
    m1, F1 = run_grad(cfg, P, ids, Gx, Gv, z, z)
    m2, F2 = run_grad(cfg, P, ids, Gx, Gv, z, z)
    assert torch.equal(F1.grad, F2.grad), "backward not deterministic"
    assert torch.equal(m1.layers[3].out_proj_x.weight.grad, m2.layers[3].out_proj_x.weight.grad)
    x0 = np.broadcast_to(P["x0"], (B, d)).astype(np.float64)
    v0 = np.broadcast_to(P["v0"], (B, d)).astype(np.float64)
    lay = [{k: a.astype(np.float64) for k, a in lp.items()} for lp in P["layers"]]
    res = O.manifold_backward(x0, v0, P["emb"][ids].astype(np.float64), lay, cfg["H"], cfg["dt"],
                              Gx.astype(np.float64), Gv.astype(np.float64))
    gclose(F1.grad.cpu(), res["forces"], "forces")
    gclose(m1.x0.grad.cpu()[0], res["x0"].sum(0), "x0")
    for l in (0, 7):
        lg, layer = res["layers"][l], m1.layers[l]
        gclose(layer.out_proj_x.weight.grad.cpu(), lg["Wx"], f"l{l} Wx")
        gclose(layer.out_proj_v.weight.grad.cpu(), lg["Wv"], f"l{l} Wv")
        gclose(torch.stack([c.forget_gate.weight.grad for c in layer.christoffels]).cpu(), lg["Wf"],
               f"l{l} Wf")
        gclose(torch.stack([c.U.grad for c in layer.christoffels]).cpu(), lg["U"], f"l{l} U")
        gclose(layer.dt_params.grad.cpu(), lg["dt_params"], f"l{l} dt")


def test_backward_c5_full_length_vs_float64_oracle():
    """C5 layer shapes over the full 1024 tokens (8 layers, 8192 reverse layer
    steps) on 2 rows: gradients vs the float64 oracle backward."""
    cfg = dict(C.CASES["c5s"], B=2, L=1024, seed=43, V=500)
    P = C.make_params(cfg)
    rng = np.random.default_rng(5)
    B, L, d = 2, 1024, cfg["d"]
    ids = rng.integers(0, cfg["V"], (B, L))
    Gx = (rng.standard_normal((B, L, d)) * 0.05).astype(np.float32)
    Gv = (rng.standard_normal((B, L, d)) * 0.05).astype(np.float32)
    z = np.zeros((B, d), np.float32)
    m, F = run_grad(cfg, P, ids, Gx, Gv, z, z)
    x0 = np.broadcast_to(P["x0"], (B, d)).astype(np.float64)
    v0 = np.broadcast_to(P["v0"], (B, d)).astype(np.float64)
    lay = [{k: a.astype(np.float64) for k, a in lp.items()} for lp in P["layers"]]
    res = O.manifold_backward(x0, v0, P["emb"][ids].astype(np.float64), lay, cfg["H"], cfg["dt"],
                              Gx.astype(np.float64), Gv.astype(np.float64))
    gclose(F.grad.cpu(), res["forces"], "forces")
    gclose(m.x0.grad.cpu()[0], res["x0"].sum(0), "x0")
    gclose(m.v0.grad.cpu()[0], res["v0"].sum(0), "v0")
    for l in (0, 4, 7):
        lg, layer = res["layers"][l], m.layers[l]
        gclose(layer.out_proj_x.weight.grad.cpu(), lg["Wx"], f"l{l} Wx")
        gclose(layer.out_proj_v.weight.grad.cpu(), lg["Wv"], f"l{l} Wv")
        gclose(torch.stack([c.forget_gate.weight.grad for c in layer.christoffels]).cpu(), lg["Wf"],
               f"l{l} Wf")
        gclose(torch.stack([c.U.grad for c in layer.christoffels]).cpu(), lg["U"], f"l{l} U")
        gclose(torch.stack([c.W.grad for c in layer.christoffels]).cpu(), lg["W"], f"l{l} W")
        gclose(layer.dt_params.grad.cpu(), lg["dt_params"], f"l{l} dt")


def test_mlayer_step_gradients_flow():
    """MLayer.forward under autograd runs the fused single-step kernels."""
    import manifold_b200 as gfn
    torch.manual_seed(0)
    layer = gfn.MLayer(64, heads=4, rank=16, base_dt=0.1, integrator_type="leapfrog").cuda()
    x = torch.randn(5, 64, device="cuda", requires_grad=True)
    v = torch.randn(5, 64, device="cuda", requires_grad=True)
    f = torch.randn(5, 64, device="cuda")
    xn, vn, _, _ = layer(x, v, f)
    (xn.sum() + 2 * vn.sum()).backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()
    assert layer.out_proj_x.weight.grad is not None


@pytest.mark.parametrize("name", list(C.GENERIC_GRAD_CASES))
def test_generic_backward_matches_reference_autograd(name):
    """Training on the generic layer step (the torus with the leapfrog
    autograd operator; Heun, RK4, Omelyan through the scheme arithmetic with
    autograd): gradients of forces, initial state, dt_params, U / W, the
    forget gates and the mixing against the reference's autograd."""
    cfg = C.GENERIC_GRAD_CASES[name]
    g = dict(np.load(os.path.join(GOLD, f"{name}.npz")))
    P = C.make_params(cfg)
    m, F = run_grad(cfg, P, g["ids"], g["Gx"], g["Gv"], g["gxf"], g["gvf"])
    assert m.layers[0].training_generic()
    gclose(F.grad.cpu(), g["g_forces"], "forces")
    gclose(m.x0.grad.cpu()[0], g["g_x0"], "x0")
    gclose(m.v0.grad.cpu()[0], g["g_v0"], "v0")
    for l, layer in enumerate(m.layers):
        gclose(layer.dt_params.grad.cpu(), g[f"l{l}_dt_params"], f"l{l} dt_params")
        gclose(torch.stack([c.forget_gate.weight.grad for c in layer.christoffels]).cpu(), g[f"l{l}_Wf"],
               f"l{l} Wf")
        gclose(torch.stack([c.forget_gate.bias.grad for c in layer.christoffels]).cpu(), g[f"l{l}_bf"],
               f"l{l} bf")
        if f"l{l}_U" in g:
            gclose(torch.stack([c.U.grad for c in layer.christoffels]).cpu(), g[f"l{l}_U"], f"l{l} U")
            gclose(torch.stack([c.W.grad for c in layer.christoffels]).cpu(), g[f"l{l}_W"], f"l{l} W")
        if cfg["H"] > 1:
            for nm in ("x", "v"):
                gclose(getattr(layer, "out_proj_" + nm).weight.grad.cpu(), g[f"l{l}_W{nm}"], f"l{l} W{nm}")
                gclose(getattr(layer, "out_proj_" + nm).bias.grad.cpu(), g[f"l{l}_b{nm}"], f"l{l} b{nm}")
            gclose(layer.mixed_norm_v.weight.grad.cpu(), g[f"l{l}_gv"], f"l{l} gv")
            if f"l{l}_gx" in g:
                gclose(layer.mixed_norm_x.weight.grad.cpu(), g[f"l{l}_gx"], f"l{l} gx")
        if f"l{l}_V" in g:
            gclose(torch.stack([c.V.weight.grad for c in layer.christoffels]).cpu(), g[f"l{l}_V"], f"l{l} V")
        if f"l{l}_gate_W1" in g:
            gclose(torch.stack([q.curvature_net[0].weight.grad for q in layer.gatings]).cpu(),
                   g[f"l{l}_gate_W1"], f"l{l} gate W1")
            gclose(torch.stack([q.curvature_net[2].bias.grad for q in layer.gatings]).cpu(),
                   g[f"l{l}_gate_b2"], f"l{l} gate b2")
        if f"l{l}_ctx_W" in g:
            gclose(layer.context_proj.weight.grad.cpu(), g[f"l{l}_ctx_W"], f"l{l} context_proj")
