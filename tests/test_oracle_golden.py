"""Pin the numpy oracle against fixtures recorded from the reference itself.

CPU only.  Tolerances are the per-step fp32 parity bar (1e-5 relative,
1e-6 absolute) scaled for sequence length where states compound.
"""
import os

import numpy as np
import pytest

from oracle import gfn_oracle as O
from tests.golden import cases as C
from tests.parity import rowwise_close

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, f"{name}.npz")))


def close(a, b, rtol, atol):
    np.testing.assert_allclose(a, b, rtol=rtol, atol=atol)


SMALL = ["tiny", "h1", "mask", "c1", "c2s", "c3s", "c4s", "c5s"]


@pytest.mark.parametrize("name", SMALL)
def test_oracle_sequence_matches_reference(name):
    cfg = C.CASES[name]
    P = C.make_params(cfg)
    g = load(name)
    F = C.oracle_forces(P, g["ids"])
    B = cfg["B"]
    x0 = np.broadcast_to(P["x0"], (B, cfg["d"])).copy()
    v0 = np.broadcast_to(P["v0"], (B, cfg["d"])).copy()
    xs, vs, x, v = O.manifold_forward(x0, v0, F, P["layers"], cfg["H"], cfg["dt"], g.get("mask"))
    close(xs, g["x_seq"], 1e-4, 1e-5)
    close(vs, g["v_seq"], 1e-4, 1e-5)
    close(x, g["x_final"], 1e-4, 1e-5)
    close(v, g["v_final"], 1e-4, 1e-5)


def test_oracle_fp64_tracks_reference_fp64():
    cfg = C.CASES["tiny"]
    P = C.make_params(cfg)
    g = load("tiny")
    P64 = dict(x0=P["x0"].astype(np.float64), v0=P["v0"].astype(np.float64),
               layers=[{k: a.astype(np.float64) for k, a in lp.items()} for lp in P["layers"]])
    F = P["emb"].astype(np.float64)[g["ids"]]
    B, d = cfg["B"], cfg["d"]
    xs, vs, _, _ = O.manifold_forward(np.broadcast_to(P64["x0"], (B, d)).copy(),
                                      np.broadcast_to(P64["v0"], (B, d)).copy(),
                                      F, P64["layers"], cfg["H"], cfg["dt"])
    close(xs, g["x_seq64"], 1e-10, 1e-12)
    close(vs, g["v_seq64"], 1e-10, 1e-12)


@pytest.mark.parametrize("name", ["c2s", "c3s", "c4s"])
def test_oracle_layer_step_matches_reference(name):
    cfg = C.CASES[name]
    g = load(name)
    P = C.make_params(cfg)
    lp = P["layers"][int(g["step_layer"])]
    xo, vo = O.mlayer_step(g["step_x"], g["step_v"], g["step_F"], lp, cfg["H"], cfg["dt"])
    rowwise_close(xo, g["step_xo"], what="x")
    rowwise_close(vo, g["step_vo"], what="v")


def test_oracle_functional_embedding_matches_reference():
    cfg = C.CASES["c3s"]
    P = C.make_params(cfg)
    g = load("c3s")
    F = O.functional_embedding(g["ids"], P["func"])
    close(F, g["forces"], 1e-5, 1e-6)


def test_oracle_units_match_reference():
    g = load("units")
    gam = O.christoffel(g["ch_v"], g["ch_U"], g["ch_W"])
    close(gam, g["ch_gamma"], 1e-5, 1e-6)
    xn, vn = O.leapfrog_head_step(g["lf_x"], g["ch_v"], g["lf_F"], g["ch_U"], g["ch_W"],
                                  g["lf_Wf"], g["lf_bf"], 0.1, g["lf_scale"], steps=3)
    close(xn, g["lf_xn"], 1e-5, 1e-6)
    close(vn, g["lf_vn"], 1e-5, 1e-6)
    for L in (20, 100):
        y = O.parallel_scan(g[f"scan{L}_a"], g[f"scan{L}_x"])
        close(y, g[f"scan{L}_y"], 1e-5, 1e-6)
        ys = O.scan_sequential(g[f"scan{L}_a"].astype(np.float64), g[f"scan{L}_x"].astype(np.float64))
        close(ys, g[f"scan{L}_y"], 1e-5, 1e-5)
    pp = {k[3:]: g[k] for k in g if k.startswith("pl_") and k not in ("pl_f", "pl_x", "pl_v")}
    xs, vs = O.parallel_mlayer(g["pl_f"], pp, heads=4)
    close(xs, g["pl_x"], 1e-5, 1e-5)
    close(vs, g["pl_v"], 1e-5, 1e-5)


def test_oracle_single_head_ops_match_reference():
    """The gated / toroidal leapfrog and the toroidal Gamma of the oracle
    against the reference's own outputs (tests/golden/ops.npz)."""
    g = load("ops")
    rowwise_close(O.torus_christoffel(g["lr_v"], g["tor_x"]), g["tor_gamma"], what="torus gamma")
    rowwise_close(O.christoffel(g["lr_v"], g["lr_U"], g["lr_W"]), g["lr_gamma"], what="low-rank gamma")
    xn, vn = O.leapfrog_head_step_gated(g["ig_x"], g["lr_v"], g["ig_F"], g["lr_U"], g["lr_W"],
                                        g["ig_Wf"], g["ig_bf"], g["ig_Wi"], 0.1, np.float32(0.87), 2)
    rowwise_close(xn, g["ig_xn"], what="input-gate leapfrog x")
    rowwise_close(vn, g["ig_vn"], what="input-gate leapfrog v")
    xn, vn = O.leapfrog_head_step_gated(g["ig_x"], g["lr_v"], g["ig_F"], g["lr_U"], g["lr_W"],
                                        g["ig_Wf"], g["ig_bf"], None, 0.1, np.float32(1.13), 3)
    rowwise_close(xn, g["st_xn"], what="stacked leapfrog x")
    rowwise_close(vn, g["st_vn"], what="stacked leapfrog v")
    xn, vn = O.leapfrog_head_step_gated(g["tor_x"], g["lr_v"], g["ig_F"], None, None, g["tl_Wf"],
                                        g["ig_bf"], None, 0.1, np.float32(0.95), 2, topology=1)
    rowwise_close(xn, g["tl_xn"], what="torus leapfrog x")
    rowwise_close(vn, g["tl_vn"], what="torus leapfrog v")


@pytest.mark.parametrize("name", C.VARIANT_CASES)
def test_oracle_generic_variants_match_reference(name):
    """The other integrators and the torus, whole model, against the reference."""
    cfg = C.CASES[name]
    P = C.make_params(cfg)
    g = load(name)
    F = C.oracle_forces(P, g["ids"])
    B = cfg["B"]
    x0 = np.broadcast_to(P["x0"], (B, cfg["d"])).copy()
    v0 = np.broadcast_to(P["v0"], (B, cfg["d"])).copy()
    xs, vs, x, v = O.manifold_forward_generic(x0, v0, F, P["layers"], cfg["H"], cfg["dt"],
                                              cfg.get("integrator", "leapfrog"), 1 if cfg.get("torus") else 0,
                                              cfg.get("active"))
    close(xs, g["x_seq"], 1e-4, 1e-5)
    close(vs, g["v_seq"], 1e-4, 1e-5)


@pytest.mark.parametrize("scheme", ["euler", "heun", "rk4", "verlet", "yoshida", "forest_ruth", "omelyan", "rk45"])
@pytest.mark.parametrize("topology", [0, 1])
def test_training_scheme_arithmetic_matches_oracle(scheme, topology):
    """The differentiable [B, H, hd] scheme arithmetic the generic layer step
    trains with equals the oracle's per-head integrator (float64, CPU)."""
    import torch
    from manifold_b200.integrators import scheme_step_torch
    rng = np.random.default_rng(11)
    B, H, hd, r = 3, 2, 8, 4
    x = rng.uniform(0, 6, (B, H, hd)) if topology else rng.standard_normal((B, H, hd))
    v = rng.standard_normal((B, H, hd))
    F = rng.standard_normal((B, H, hd))
    U = rng.standard_normal((H, hd, r)) * 0.3
    W = rng.standard_normal((H, hd, r)) * 0.3
    fin = 2 * hd if topology else hd
    Wf = rng.standard_normal((H, hd, fin)) * 0.1
    bf = rng.standard_normal((H, hd)) * 0.3
    Wi = rng.standard_normal((H, hd, hd)) * 0.1
    sc = np.array([0.9, 1.1])
    T = torch.as_tensor
    xt, vt = scheme_step_torch(scheme, T(x), T(v), T(F), None if topology else T(U), None if topology else T(W),
                               T(Wf), T(bf), T(Wi), T(0.1 * sc).view(1, H, 1), topology)
    for h in range(H):
        xo, vo = O.integrator_step(scheme, x[:, h], v[:, h], F[:, h], None if topology else U[h],
                                   None if topology else W[h], Wf[h], bf[h], Wi[h], 0.1, sc[h], 1, topology)
        np.testing.assert_allclose(xt[:, h].numpy(), xo, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(vt[:, h].numpy(), vo, rtol=1e-12, atol=1e-12)
