"""Seeded parity cases shared by the golden generator and the tests.

Weights are drawn here from numpy's PCG64 (bit-stable across machines) in the
canonical layout the oracle uses, then loaded into the reference model by
``make_golden.py`` and into ``manifold_b200`` by the GPU tests, so both run on
identical parameters.  Fixtures therefore store only inputs and outputs.

Shapes follow the benchmark configurations (C1..C5): C1 is complete; the
larger ones are short slices (few rows/tokens) with the full layer shapes.
"""
import math
import numpy as np

# name -> config.  rank is the model-level rank; the per-head rank is
# max(4, rank // heads) as in the reference's MLayer.
CASES = {
    "tiny":  dict(V=5, d=32, NL=2, H=2, rank=8, B=3, L=5, dt=0.1, seed=1),
    "h1":    dict(V=4, d=16, NL=2, H=1, rank=4, B=2, L=4, dt=0.1, seed=2),
    "mask":  dict(V=7, d=64, NL=3, H=4, rank=16, B=4, L=6, dt=0.05, seed=3, mask=True),
    "c1":    dict(V=2, d=128, NL=4, H=4, rank=16, B=32, L=20, dt=0.1, seed=11, parity=True),
    "c2s":   dict(V=2, d=256, NL=6, H=8, rank=32, B=4, L=6, dt=0.1, seed=12, parity=True),
    "c3s":   dict(V=50257, d=512, NL=12, H=8, rank=32, B=2, L=3, dt=0.1, seed=13, functional=True),
    "c4s":   dict(V=32000, d=1024, NL=24, H=16, rank=64, B=3, L=1, dt=0.1, seed=14),
    "c5s":   dict(V=32000, d=512, NL=8, H=8, rank=32, B=2, L=4, dt=0.1, seed=15),
    # other integrators and the torus (model path of the multi-scheme kernel)
    "heun_s":   dict(V=6, d=32, NL=2, H=2, rank=8, B=3, L=4, dt=0.1, seed=41, integrator="heun"),
    "rk4_s":    dict(V=6, d=64, NL=2, H=4, rank=16, B=2, L=3, dt=0.1, seed=42, integrator="rk4"),
    "euler_s":  dict(V=6, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=45, integrator="euler"),
    "verlet_s": dict(V=6, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=46, integrator="verlet"),
    "yoshida_s": dict(V=6, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=47, integrator="yoshida"),
    "forest_ruth_s": dict(V=6, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=48,
                          integrator="forest_ruth"),
    "omelyan_s": dict(V=6, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=49, integrator="omelyan"),
    "rk45_s":   dict(V=6, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=50, integrator="rk45"),
    "torus_s":  dict(V=6, d=32, NL=2, H=2, rank=8, B=3, L=4, dt=0.1, seed=43, torus=True),
    "torus_heun_s": dict(V=6, d=64, NL=2, H=4, rank=16, B=2, L=3, dt=0.1, seed=44, torus=True,
                         integrator="heun"),
    "torus_h1": dict(V=5, d=16, NL=2, H=1, rank=4, B=2, L=4, dt=0.1, seed=51, torus=True),
    # active inference (reactive curvature, singularities, dynamic time, recursive geodesics)
    "ai_heun_s": dict(V=6, d=32, NL=2, H=2, rank=8, B=3, L=4, dt=0.1, seed=52, integrator="heun",
                      active={"enabled": True, "reactive_curvature": {"enabled": True, "plasticity": 0.5},
                              "singularities": {"enabled": True, "threshold": 0.5, "strength": 3.0}}),
    "ai_torus_s": dict(V=6, d=32, NL=2, H=2, rank=8, B=3, L=4, dt=0.1, seed=53, torus=True,
                       active={"enabled": True, "reactive_curvature": {"enabled": True, "plasticity": 0.2},
                               "singularities": {"enabled": True, "threshold": 0.55, "strength": 2.0}}),
    "dyn_s": dict(V=6, d=64, NL=2, H=4, rank=16, B=3, L=4, dt=0.1, seed=54,
                  active={"dynamic_time": {"enabled": True}, "recursive_geodesics": {"enabled": True}}),
    "dyn_rk4_torus_s": dict(V=6, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=55, torus=True,
                            integrator="rk4", active={"dynamic_time": {"enabled": True}}),
}
VARIANT_CASES = ["heun_s", "rk4_s", "euler_s", "verlet_s", "yoshida_s", "forest_ruth_s", "omelyan_s",
                 "rk45_s", "torus_s", "torus_heun_s", "torus_h1", "ai_heun_s", "ai_torus_s", "dyn_s",
                 "dyn_rk4_torus_s"]

# Gradient (BPTT) cases: upstream gradients on x_seq, v_seq and the final
# state, gradients taken by the reference's autograd.  "gc5" has the C5 layer
# shapes; its d x d mixing-weight gradients are stored as row/column sums.
GRAD_CASES = {
    "gsmall": dict(V=7, d=32, NL=2, H=2, rank=8, B=3, L=4, dt=0.1, seed=31),
    "gh1":    dict(V=5, d=16, NL=2, H=1, rank=4, B=2, L=3, dt=0.1, seed=32),
    "gmask":  dict(V=7, d=64, NL=3, H=4, rank=16, B=4, L=6, dt=0.05, seed=33, mask=True),
    "gc5":    dict(V=300, d=512, NL=2, H=8, rank=32, B=2, L=3, dt=0.1, seed=34),
}
# gradient cases of the generic (layer-by-layer) path
GENERIC_GRAD_CASES = {
    "gtorus": dict(V=7, d=32, NL=2, H=2, rank=8, B=3, L=4, dt=0.1, seed=36, torus=True),
    "gtorus_h1": dict(V=5, d=16, NL=2, H=1, rank=4, B=2, L=3, dt=0.1, seed=37, torus=True),
    "gheun": dict(V=7, d=32, NL=2, H=2, rank=8, B=3, L=4, dt=0.1, seed=38, integrator="heun"),
    "grk4_torus": dict(V=7, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=39, integrator="rk4", torus=True),
    "gomelyan": dict(V=7, d=32, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=40, integrator="omelyan"),
    "gai_heun": dict(V=7, d=32, NL=2, H=2, rank=8, B=3, L=3, dt=0.1, seed=56, integrator="heun",
                     active={"enabled": True, "reactive_curvature": {"enabled": True, "plasticity": 0.5},
                             "singularities": {"enabled": True, "threshold": 0.5, "strength": 3.0}}),
    "gai_torus": dict(V=7, d=32, NL=2, H=2, rank=8, B=3, L=3, dt=0.1, seed=57, torus=True,
                      active={"enabled": True, "reactive_curvature": {"enabled": True, "plasticity": 0.2}}),
    "ghd128": dict(V=7, d=256, NL=2, H=2, rank=8, B=2, L=3, dt=0.1, seed=59),
    "gdyn": dict(V=7, d=64, NL=2, H=4, rank=16, B=3, L=3, dt=0.1, seed=58,
                 active={"dynamic_time": {"enabled": True}, "recursive_geodesics": {"enabled": True}}),
}


def head_rank(cfg):
    return max(4, cfg["rank"] // cfg["H"])


def dt_param_init(dt, H):
    """The reference's per-head dt init: log(expm1(dt/0.9)) + 0.1*i."""
    base = math.log(math.expm1(dt / 0.9))
    return np.array([base + 0.1 * i for i in range(H)], np.float32)


def make_layer_params(rng, d, H, r, dt, torus=False):
    hd = d // H
    f = np.float32
    if torus:
        # ToroidalChristoffel: the gate reads [sin x, cos x]; the x mixer reads
        # [sin x, cos x, tanh(v / 100)]; no U / W
        return dict(
            Wf=(rng.standard_normal((H, hd, 2 * hd)) * 0.1).astype(f),
            bf=(rng.standard_normal((H, hd)) * 0.5).astype(f),
            Wi=(rng.standard_normal((H, hd, hd)) * 0.1).astype(f),
            dt_params=(dt_param_init(dt, H) + rng.standard_normal(H).astype(f) * 0.05).astype(f),
            Wx=(rng.standard_normal((d, 3 * d)) / math.sqrt(3 * d)).astype(f),
            bx=(rng.standard_normal(d) * 0.1).astype(f),
            gx=(1.0 + rng.standard_normal(d) * 0.1).astype(f),
            Wv=(rng.standard_normal((d, d)) / math.sqrt(d)).astype(f),
            bv=(rng.standard_normal(d) * 0.1).astype(f),
            gv=(1.0 + rng.standard_normal(d) * 0.1).astype(f),
        )
    return dict(
        U=(rng.standard_normal((H, hd, r)) * 0.2).astype(f),
        W=(rng.standard_normal((H, hd, r)) * 0.2).astype(f),
        Wf=(rng.standard_normal((H, hd, hd)) * 0.1).astype(f),
        bf=(rng.standard_normal((H, hd)) * 0.5).astype(f),
        Wi=(rng.standard_normal((H, hd, hd)) * 0.1).astype(f),  # input_gate: unused by leapfrog
        dt_params=(dt_param_init(dt, H) + rng.standard_normal(H).astype(f) * 0.05).astype(f),
        Wx=(rng.standard_normal((d, d)) / math.sqrt(d)).astype(f),
        bx=(rng.standard_normal(d) * 0.1).astype(f),
        gx=(1.0 + rng.standard_normal(d) * 0.1).astype(f),
        Wv=(rng.standard_normal((d, d)) / math.sqrt(d)).astype(f),
        bv=(rng.standard_normal(d) * 0.1).astype(f),
        gv=(1.0 + rng.standard_normal(d) * 0.1).astype(f),
    )


def make_functional_params(rng, d, coord_dim=16, hidden=64, omega_0=30.0):
    f = np.float32
    p = {}
    p["W0"] = rng.uniform(-1 / coord_dim, 1 / coord_dim, (hidden, coord_dim)).astype(f)
    p["b0"] = rng.uniform(-0.25, 0.25, hidden).astype(f)
    bound = math.sqrt(6 / hidden) / omega_0
    for i in (1, 2):
        p[f"W{i}"] = rng.uniform(-bound, bound, (hidden, hidden)).astype(f)
        p[f"b{i}"] = rng.uniform(-0.125, 0.125, hidden).astype(f)
    p["Wo"] = (rng.uniform(-1 / 8, 1 / 8, (d, hidden)) * 1.5).astype(f)
    p["bo"] = (rng.standard_normal(d) * 0.01).astype(f)
    p["impulse"] = np.array(1.25, f)
    return p


def make_params(cfg):
    """All model parameters for a case (canonical layout)."""
    rng = np.random.default_rng(cfg["seed"])
    d, H, NL = cfg["d"], cfg["H"], cfg["NL"]
    r = head_rank(cfg)
    f = np.float32
    P = dict(
        x0=(rng.standard_normal(d) * 0.02).astype(f),
        v0=(rng.standard_normal(d) * 0.01).astype(f),
        layers=[make_layer_params(rng, d, H, r, cfg["dt"], cfg.get("torus", False)) for _ in range(NL)],
    )
    if cfg.get("functional"):
        P["func"] = make_functional_params(rng, d)
    else:
        P["emb"] = rng.standard_normal((cfg["V"], d)).astype(f)
    if cfg.get("active"):
        # active-inference parameters from a separate stream (the draws above
        # stay those of the plain cases)
        ra = np.random.default_rng(cfg["seed"] + 500)
        hd = d // H
        fin = 2 * hd if cfg.get("torus") else hd
        for lp in P["layers"]:
            lp["V"] = (ra.standard_normal((H, fin)) * 0.5).astype(f)
            lp["Vb"] = (ra.standard_normal(H) * 0.3).astype(f)
            q = hd // 4
            lp["gW1"] = (ra.standard_normal((H, q, fin)) * 0.3).astype(f)
            lp["gb1"] = (ra.standard_normal((H, q)) * 0.1).astype(f)
            lp["gW2"] = (ra.standard_normal((H, 1, q)) * 0.5).astype(f)
            lp["gb2"] = (ra.standard_normal((H, 1)) * 0.5 + 1.0).astype(f)
            lp["cW"] = (ra.standard_normal((d, H)) * 0.2).astype(f)
            lp["cb"] = (ra.standard_normal(d) * 0.05).astype(f)
    return P


def zipf_ids(rng, V, shape, s=1.1):
    """Zipf(s) over ranks 1..V by inverse CDF on the finite support; rank k -> id k-1."""
    w = np.arange(1, V + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    u = rng.random(shape)
    return np.searchsorted(cdf, u, side="right").clip(0, V - 1).astype(np.int64)


def make_inputs(cfg):
    """Token ids (and mask) for a case."""
    rng = np.random.default_rng(cfg["seed"] + 1000)
    B, L, V = cfg["B"], cfg["L"], cfg["V"]
    if cfg.get("parity"):
        ids = rng.integers(0, 2, (B, L)).astype(np.int64)     # Bernoulli(0.5) bits
    elif V > 1000:
        ids = zipf_ids(rng, V, (B, L))
    else:
        ids = rng.integers(0, V, (B, L)).astype(np.int64)
    out = dict(ids=ids)
    if cfg.get("mask"):
        m = np.ones((B, L), np.float32)
        m[0, 2:] = 0.0
        m[1, 4] = 0.0
        out["mask"] = m
    return out


def oracle_forces(P, ids):
    """Force F(u_t) for the ids (lookup or functional), via the oracle."""
    from oracle import gfn_oracle as O
    if "func" in P:
        return O.functional_embedding(ids, P["func"])
    return O.embedding_lookup(ids, P["emb"])


def load_into_model(m, cfg, P):
    """Copy the canonical parameters into a Manifold whose module tree follows
    the reference's (the reference model itself or manifold_b200.Manifold)."""
    import torch

    def T(a):
        return torch.as_tensor(np.asarray(a, np.float32).copy())

    with torch.no_grad():
        dev = m.x0.device
        m.x0.copy_(T(P["x0"])[None].to(dev))
        m.v0.copy_(T(P["v0"])[None].to(dev))
        if "emb" in P:
            m.embedding.weight.copy_(T(P["emb"]).to(dev))
        else:
            fp = P["func"]
            for i in range(3):
                m.embedding.net[i].linear.weight.copy_(T(fp[f"W{i}"]).to(dev))
                m.embedding.net[i].linear.bias.copy_(T(fp[f"b{i}"]).to(dev))
            m.embedding.out_proj.weight.copy_(T(fp["Wo"]).to(dev))
            m.embedding.out_proj.bias.copy_(T(fp["bo"]).to(dev))
            m.embedding.impulse_scale.copy_(T(fp["impulse"]).to(dev))
        for layer, lp in zip(m.layers, P["layers"]):
            load_into_layer(layer, cfg, lp)


def load_into_layer(layer, cfg, lp):
    import torch

    def T(a):
        return torch.as_tensor(np.asarray(a, np.float32).copy()).to(layer.dt_params.device)

    with torch.no_grad():
        layer.dt_params.copy_(T(lp["dt_params"]))
        for h, ch in enumerate(layer.christoffels):
            if "U" in lp:
                ch.U.copy_(T(lp["U"][h]))
                ch.W.copy_(T(lp["W"][h]))
            ch.forget_gate.weight.copy_(T(lp["Wf"][h]))
            ch.forget_gate.bias.copy_(T(lp["bf"][h]))
            ch.input_gate.weight.copy_(T(lp["Wi"][h]))
        if "V" in lp:
            for h, ch in enumerate(layer.christoffels):
                if getattr(ch, "V", None) is not None:
                    ch.V.weight.copy_(T(lp["V"][h])[None])
                    if ch.V.bias is not None:
                        ch.V.bias.copy_(T(lp["Vb"][h])[None])
            for h, g in enumerate(layer.gatings):
                g.curvature_net[0].weight.copy_(T(lp["gW1"][h]))
                g.curvature_net[0].bias.copy_(T(lp["gb1"][h]))
                g.curvature_net[2].weight.copy_(T(lp["gW2"][h]))
                g.curvature_net[2].bias.copy_(T(lp["gb2"][h]))
            if getattr(layer, "context_proj", None) is not None:
                layer.context_proj.weight.copy_(T(lp["cW"]))
                layer.context_proj.bias.copy_(T(lp["cb"]))
        if cfg["H"] > 1:
            layer.out_proj_x.weight.copy_(T(lp["Wx"]))
            layer.out_proj_x.bias.copy_(T(lp["bx"]))
            layer.out_proj_v.weight.copy_(T(lp["Wv"]))
            layer.out_proj_v.bias.copy_(T(lp["bv"]))
            layer.mixed_norm_x.weight.copy_(T(lp["gx"]))
            layer.mixed_norm_v.weight.copy_(T(lp["gv"]))


def model_kwargs(cfg):
    pc = {}
    if cfg.get("functional"):
        pc = {"embedding": {"type": "functional", "mode": "binary", "coord_dim": 16}}
    if cfg.get("torus"):
        pc = dict(pc, topology={"type": "torus"})
    if cfg.get("active"):
        pc = dict(pc, active_inference=cfg["active"])
    return dict(vocab_size=cfg["V"], dim=cfg["d"], depth=cfg["NL"], rank=cfg["rank"],
                heads=cfg["H"], integrator_type=cfg.get("integrator", "leapfrog"), base_dt=cfg["dt"],
                physics_config=pc)
