"""Pin the oracle's hand-written BPTT backward against the reference's own
autograd gradients (fixtures from tests/golden/make_golden.py).  CPU only."""
import os

import numpy as np
import pytest

from oracle import gfn_oracle as O
from tests.golden import cases as C

GOLD = os.path.join(os.path.dirname(__file__), "golden")
RTOL, ATOL = 1e-3, 1e-5  # float32 gradients through L x NL steps, scaled per tensor


def gclose(a, b, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(float(np.max(np.abs(b))), 1e-30)
    err = float(np.max(np.abs(a - b)))
    assert err <= ATOL + RTOL * scale, f"{what}: max |diff| {err:.3e} vs scale {scale:.3e}"


def oracle_grads(name, dtype=np.float32):
    cfg = C.GRAD_CASES[name]
    g = dict(np.load(os.path.join(GOLD, f"{name}.npz")))
    P = C.make_params(cfg)
    B, d = cfg["B"], cfg["d"]
    cast = lambda a: np.asarray(a, dtype)
    layers = [{k: cast(v) for k, v in lp.items()} for lp in P["layers"]]
    x0 = np.broadcast_to(cast(P["x0"]), (B, d)).copy()
    v0 = np.broadcast_to(cast(P["v0"]), (B, d)).copy()
    F = cast(P["emb"][g["ids"]])
    res = O.manifold_backward(x0, v0, F, layers, cfg["H"], cfg["dt"], cast(g["Gx"]), cast(g["Gv"]),
                              cast(g["gxf"]), cast(g["gvf"]), g.get("mask"))
    return cfg, g, res


@pytest.mark.parametrize("name", list(C.GRAD_CASES))
def test_oracle_backward_matches_reference_autograd(name):
    cfg, g, res = oracle_grads(name, np.float64)
    gclose(res["forces"], g["g_forces"], "forces")
    gclose(res["x0"].sum(0), g["g_x0"], "x0")
    gclose(res["v0"].sum(0), g["g_v0"], "v0")
    for l, lg in enumerate(res["layers"]):
        for k in ("dt_params", "U", "W", "Wf", "bf"):
            gclose(lg[k], g[f"l{l}_{k}"], f"layer {l} {k}")
        if cfg["H"] > 1:
            for nm in ("x", "v"):
                if f"l{l}_W{nm}" in g:
                    gclose(lg[f"W{nm}"], g[f"l{l}_W{nm}"], f"layer {l} W{nm}")
                else:
                    gclose(lg[f"W{nm}"].sum(1), g[f"l{l}_W{nm}_rowsum"], f"layer {l} W{nm} rows")
                    gclose(lg[f"W{nm}"].sum(0), g[f"l{l}_W{nm}_colsum"], f"layer {l} W{nm} cols")
                    gclose(lg[f"W{nm}"][:16, :16], g[f"l{l}_W{nm}_corner"], f"layer {l} W{nm}")
                gclose(lg[f"b{nm}"], g[f"l{l}_b{nm}"], f"layer {l} b{nm}")
                gclose(lg[f"g{nm}"], g[f"l{l}_g{nm}"], f"layer {l} g{nm}")
