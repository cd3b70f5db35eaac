"""Generate golden fixtures by running the reference implementation itself.

Run in a container that has the reference checkout (read-only) available:

    GFN_REFERENCE=/path/to/manifold python tests/golden/make_golden.py

It imports the reference package ``gfn``, builds each case's model with the
reference's own constructors, loads the seeded canonical weights from
``cases.py`` into it, runs the reference CPU path (eval mode, no grad) and
writes ``<case>.npz`` beside this script.  The fixtures hold only inputs and
outputs; the weights are regenerated from the seed by ``cases.make_params``.

This script is the only thing in the repository that touches the reference;
the fixtures it wrote are committed, and nothing at test time reads the
reference.
"""
import contextlib
import io
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
REF = os.environ.get("GFN_REFERENCE")
if not REF:
    sys.exit("set GFN_REFERENCE to the directory holding the reference's `gfn` package")
sys.path.append(REF)

from tests.golden import cases as C  # noqa: E402

with contextlib.redirect_stdout(io.StringIO()), contextlib.redirect_stderr(io.StringIO()):
    import gfn  # noqa: E402
    from gfn.model import Manifold  # noqa: E402
    from gfn.integrators import LeapfrogIntegrator  # noqa: E402
    from gfn.geometry import LowRankChristoffel, ToroidalChristoffel  # noqa: E402
    from gfn.layers import ParallelMLayer  # noqa: E402
    from gfn.scan import parallel_scan  # noqa: E402


def T(a):
    a = np.asarray(a)
    return torch.from_numpy(a.copy()) if a.ndim == 0 else torch.from_numpy(np.ascontiguousarray(a))


def build_reference(cfg, P):
    with contextlib.redirect_stdout(io.StringIO()):
        m = Manifold(**C.model_kwargs(cfg))
    C.load_into_model(m, cfg, P)
    return m.eval()


def run_model(m, ids, mask=None, state=None):
    with torch.no_grad():
        out = m(input_ids=T(ids), attention_mask=None if mask is None else T(mask), state=state)
    _, (x, v), _, v_seq, x_seq, forces = out
    return dict(x_seq=torch.stack(x_seq, 1).numpy(), v_seq=torch.stack(v_seq, 1).numpy(),
                x_final=x.numpy(), v_final=v.numpy(), forces=forces.numpy())


def gen_model_case(name, cfg):
    P = C.make_params(cfg)
    inp = C.make_inputs(cfg)
    m = build_reference(cfg, P)
    res = run_model(m, inp["ids"], inp.get("mask"))
    out = dict(ids=inp["ids"], x_seq=res["x_seq"], v_seq=res["v_seq"],
               x_final=res["x_final"], v_final=res["v_final"])
    if "mask" in inp:
        out["mask"] = inp["mask"]
    if cfg.get("functional"):
        out["forces"] = res["forces"]
    if name in ("c1", "tiny"):
        # float64 run of the same model: the drift reference.
        m64 = m.double()
        r64 = run_model(m64, inp["ids"], inp.get("mask"))
        out["x_seq64"] = r64["x_seq"]
        out["v_seq64"] = r64["v_seq"]
    if name == "c4s":
        # streaming decode: continue one more token from the returned state
        rng = np.random.default_rng(99)
        ids2 = rng.integers(0, cfg["V"], (cfg["B"], 1)).astype(np.int64)
        st = (T(res["x_final"]), T(res["v_final"]))
        r2 = run_model(m, ids2, state=st)
        out["ids2"] = ids2
        out["x_final2"] = r2["x_final"]
        out["v_final2"] = r2["v_final"]
    if name in ("c4s", "c2s", "c3s"):
        # teacher-forced single layer step from a random state (per-step parity)
        rng = np.random.default_rng(cfg["seed"] + 7)
        B, d = 5, cfg["d"]
        xs = rng.standard_normal((B, d)).astype(np.float32)
        vs = (rng.standard_normal((B, d)) * 3).astype(np.float32)
        Fs = rng.standard_normal((B, d)).astype(np.float32)
        li = cfg["NL"] // 2
        with torch.no_grad():
            xo, vo, _, _ = m.layers[li](T(xs), T(vs), T(Fs))
        out.update(step_layer=np.array(li), step_x=xs, step_v=vs, step_F=Fs,
                   step_xo=xo.numpy(), step_vo=vo.numpy())
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(name, {k: v.shape for k, v in out.items()})


def gen_units():
    """Unit-level goldens: Christoffel, per-head leapfrog, scans, ParallelMLayer."""
    rng = np.random.default_rng(2024)
    out = {}
    # LowRankChristoffel with friction returned separately (leapfrog usage)
    hd, r, B = 24, 4, 7
    ch = LowRankChristoffel(hd, r)
    U = (rng.standard_normal((hd, r)) * 0.5).astype(np.float32)
    W = (rng.standard_normal((hd, r)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, hd)) * 4).astype(np.float32)
    x = rng.standard_normal((B, hd)).astype(np.float32)
    with torch.no_grad():
        ch.U.copy_(T(U)); ch.W.copy_(T(W))
        ch.return_friction_separately = True
        g, _ = ch(T(v), T(x))
    out.update(ch_U=U, ch_W=W, ch_v=v, ch_gamma=g.numpy())
    # LeapfrogIntegrator, 3 steps, with friction weights
    Wf = (rng.standard_normal((hd, hd)) * 0.2).astype(np.float32)
    bf = (rng.standard_normal(hd) * 0.5).astype(np.float32)
    F = rng.standard_normal((B, hd)).astype(np.float32)
    integ = LeapfrogIntegrator(ch, dt=0.1)
    scale = torch.tensor(0.87)
    with torch.no_grad():
        xn, vn = integ(T(x), T(v), force=T(F), dt_scale=scale, steps=3,
                       W_forget_stack=T(Wf)[None], W_input_stack=T(Wf)[None] * 0,
                       b_forget_stack=T(bf)[None], topology=0)
    out.update(lf_x=x, lf_Wf=Wf, lf_bf=bf, lf_F=F, lf_scale=np.float32(0.87),
               lf_xn=xn.numpy(), lf_vn=vn.numpy())
    # parallel_scan: short (sequential branch) and long (doubling branch)
    for L in (20, 100):
        a = rng.uniform(0.5, 1.0, (3, L, 8)).astype(np.float32)
        xx = rng.standard_normal((3, L, 8)).astype(np.float32)
        with torch.no_grad():
            y = parallel_scan(T(a), T(xx))
        out[f"scan{L}_a"] = a; out[f"scan{L}_x"] = xx; out[f"scan{L}_y"] = y.numpy()
    # ParallelMLayer with seeded torch init; record its weights (small)
    torch.manual_seed(5)
    D, H, B, L = 32, 4, 2, 40
    pl = ParallelMLayer(D, heads=H)
    f = rng.standard_normal((B, L, D)).astype(np.float32)
    with torch.no_grad():
        xs, vs, _, _ = pl(None, None, T(f))
    out.update(pl_f=f, pl_x=xs.numpy(), pl_v=vs.numpy(),
               pl_ln_w=pl.norm_x.weight.detach().numpy(), pl_ln_b=pl.norm_x.bias.detach().numpy(),
               pl_WA=pl.to_A[0].weight.detach().numpy(), pl_bA=pl.to_A[0].bias.detach().numpy(),
               pl_Wdt=pl.to_dt[0].weight.detach().numpy(), pl_bdt=pl.to_dt[0].bias.detach().numpy(),
               pl_WB=pl.to_B.weight.detach().numpy(), pl_bB=pl.to_B.bias.detach().numpy())
    np.savez_compressed(os.path.join(HERE, "units.npz"), **out)
    print("units", len(out))


def _leaf(a):
    return T(a).clone().requires_grad_(True)


def gen_ops():
    """Goldens of the single-head operators with their reference autograd
    gradients: the low-rank and toroidal Christoffel terms, and the leapfrog
    integrator with the Christoffel's own gates (input gate included), with
    explicit forget stacks, and on the torus."""
    rng = np.random.default_rng(77)
    out = {}
    hd, r, B = 32, 8, 9
    # low-rank Gamma and its gradients
    U = (rng.standard_normal((hd, r)) * 0.4).astype(np.float32)
    W = (rng.standard_normal((hd, r)) * 0.4).astype(np.float32)
    v = (rng.standard_normal((B, hd)) * 3).astype(np.float32)
    G = rng.standard_normal((B, hd)).astype(np.float32)
    ch = LowRankChristoffel(hd, r)
    with torch.no_grad():
        ch.U.copy_(T(U)); ch.W.copy_(T(W))
    ch.return_friction_separately = True
    vv = _leaf(v)
    g, _ = ch(vv, torch.zeros(B, hd))
    (g * T(G)).sum().backward()
    out.update(lr_U=U, lr_W=W, lr_v=v, lr_G=G, lr_gamma=g.detach().numpy(), lr_dv=vv.grad.numpy(),
               lr_dU=ch.U.grad.numpy(), lr_dW=ch.W.grad.numpy())
    # toroidal Gamma and its gradients
    tc = ToroidalChristoffel(hd, physics_config={"topology": {"type": "torus", "major_radius": 2.0,
                                                              "minor_radius": 1.0}})
    tc.return_friction_separately = True
    xt = rng.uniform(0, 2 * np.pi, (B, hd)).astype(np.float32)
    xx, vv = _leaf(xt), _leaf(v)
    g, _ = tc(vv, xx)
    (g * T(G)).sum().backward()
    out.update(tor_x=xt, tor_gamma=g.detach().numpy(), tor_dv=vv.grad.numpy(), tor_dx=xx.grad.numpy())
    # leapfrog, the Christoffel's own gates (forget + input gate), 2 steps
    x = rng.standard_normal((B, hd)).astype(np.float32)
    F = rng.standard_normal((B, hd)).astype(np.float32)
    Gx = rng.standard_normal((B, hd)).astype(np.float32)
    Gv = rng.standard_normal((B, hd)).astype(np.float32)
    Wf = (rng.standard_normal((hd, hd)) * 0.2).astype(np.float32)
    bf = (rng.standard_normal(hd) * 0.5).astype(np.float32)
    Wi = (rng.standard_normal((hd, hd)) * 0.2).astype(np.float32)
    ch = LowRankChristoffel(hd, r)
    with torch.no_grad():
        ch.U.copy_(T(U)); ch.W.copy_(T(W))
        ch.forget_gate.weight.copy_(T(Wf)); ch.forget_gate.bias.copy_(T(bf))
        ch.input_gate.weight.copy_(T(Wi))
    integ = LeapfrogIntegrator(ch, dt=0.1)
    xx, vv, ff = _leaf(x), _leaf(v), _leaf(F)
    xn, vn = integ(xx, vv, force=ff, dt_scale=torch.tensor(0.87), steps=2)
    ((xn * T(Gx)).sum() + (vn * T(Gv)).sum()).backward()
    out.update(ig_x=x, ig_F=F, ig_Gx=Gx, ig_Gv=Gv, ig_Wf=Wf, ig_bf=bf, ig_Wi=Wi,
               ig_xn=xn.detach().numpy(), ig_vn=vn.detach().numpy(), ig_dx=xx.grad.numpy(),
               ig_dv=vv.grad.numpy(), ig_dF=ff.grad.numpy(), ig_dU=ch.U.grad.numpy(),
               ig_dW=ch.W.grad.numpy(), ig_dWf=ch.forget_gate.weight.grad.numpy(),
               ig_dbf=ch.forget_gate.bias.grad.numpy(), ig_dWi=ch.input_gate.weight.grad.numpy())
    # leapfrog with explicit forget stacks (the MLayer usage), 3 steps
    ch = LowRankChristoffel(hd, r)
    with torch.no_grad():
        ch.U.copy_(T(U)); ch.W.copy_(T(W))
    integ = LeapfrogIntegrator(ch, dt=0.1)
    xx, vv, ff = _leaf(x), _leaf(v), _leaf(F)
    wf, bb = _leaf(Wf[None]), _leaf(bf[None])
    xn, vn = integ(xx, vv, force=ff, dt_scale=torch.tensor(1.13), steps=3, W_forget_stack=wf,
                   b_forget_stack=bb, topology=0)
    ((xn * T(Gx)).sum() + (vn * T(Gv)).sum()).backward()
    out.update(st_xn=xn.detach().numpy(), st_vn=vn.detach().numpy(), st_dx=xx.grad.numpy(),
               st_dv=vv.grad.numpy(), st_dF=ff.grad.numpy(), st_dU=ch.U.grad.numpy(),
               st_dW=ch.W.grad.numpy(), st_dWf=wf.grad[0].numpy(), st_dbf=bb.grad[0].numpy())
    # toroidal leapfrog with a forget stack over [sin x, cos x], 2 steps
    tc = ToroidalChristoffel(hd, physics_config={"topology": {"type": "torus"}})
    Wft = (rng.standard_normal((hd, 2 * hd)) * 0.2).astype(np.float32)
    integ = LeapfrogIntegrator(tc, dt=0.1)
    xx, vv, ff = _leaf(xt), _leaf(v), _leaf(F)
    wf, bb = _leaf(Wft[None]), _leaf(bf[None])
    xn, vn = integ(xx, vv, force=ff, dt_scale=torch.tensor(0.95), steps=2, W_forget_stack=wf,
                   b_forget_stack=bb, topology=1)
    ((xn * T(Gx)).sum() + (vn * T(Gv)).sum()).backward()
    out.update(tl_Wf=Wft, tl_xn=xn.detach().numpy(), tl_vn=vn.detach().numpy(), tl_dx=xx.grad.numpy(),
               tl_dv=vv.grad.numpy(), tl_dF=ff.grad.numpy(), tl_dWf=wf.grad[0].numpy(),
               tl_dbf=bb.grad[0].numpy())
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **out)
    print("ops", len(out))


def gen_grad_case(name, cfg):
    """Reference autograd gradients of <Gx, x_seq> + <Gv, v_seq> + <gx, x_L> + <gv, v_L>."""
    P = C.make_params(cfg)
    inp = C.make_inputs(cfg)
    m = build_reference(cfg, P).train()
    rng = np.random.default_rng(cfg["seed"] + 5)
    B, L, d = cfg["B"], cfg["L"], cfg["d"]
    Gx = rng.standard_normal((B, L, d)).astype(np.float32)
    Gv = rng.standard_normal((B, L, d)).astype(np.float32)
    gxf = rng.standard_normal((B, d)).astype(np.float32)
    gvf = rng.standard_normal((B, d)).astype(np.float32)
    F = T(P["emb"][inp["ids"]]).requires_grad_(True)
    mask = T(inp["mask"]) if "mask" in inp else None
    with contextlib.redirect_stdout(io.StringIO()):
        _, (x, v), _, v_seq, x_seq, _ = m(force_manual=F, attention_mask=mask)
    loss = (torch.stack(x_seq, 1) * T(Gx)).sum() + (torch.stack(v_seq, 1) * T(Gv)).sum() \
        + (x * T(gxf)).sum() + (v * T(gvf)).sum()
    loss.backward()
    out = dict(ids=inp["ids"], Gx=Gx, Gv=Gv, gxf=gxf, gvf=gvf, g_forces=F.grad.numpy(),
               g_x0=m.x0.grad.numpy()[0], g_v0=m.v0.grad.numpy()[0],
               x_seq=torch.stack(x_seq, 1).detach().numpy())
    if "mask" in inp:
        out["mask"] = inp["mask"]
    big = name == "gc5"
    for l, layer in enumerate(m.layers):
        out[f"l{l}_dt_params"] = layer.dt_params.grad.numpy()
        if not cfg.get("torus"):
            out[f"l{l}_U"] = np.stack([c.U.grad.numpy() for c in layer.christoffels])
            out[f"l{l}_W"] = np.stack([c.W.grad.numpy() for c in layer.christoffels])
        out[f"l{l}_Wf"] = np.stack([c.forget_gate.weight.grad.numpy() for c in layer.christoffels])
        out[f"l{l}_bf"] = np.stack([c.forget_gate.bias.grad.numpy() for c in layer.christoffels])
        if cfg["H"] > 1:
            for nm, mod in (("x", "out_proj_x"), ("v", "out_proj_v")):
                gW = getattr(layer, mod).weight.grad.numpy()
                if big:
                    out[f"l{l}_W{nm}_rowsum"] = gW.sum(1)
                    out[f"l{l}_W{nm}_colsum"] = gW.sum(0)
                    out[f"l{l}_W{nm}_corner"] = gW[:16, :16]
                else:
                    out[f"l{l}_W{nm}"] = gW
                out[f"l{l}_b{nm}"] = getattr(layer, mod).bias.grad.numpy()
                gn = getattr(layer, "mixed_norm_" + nm).weight.grad
                if gn is not None:  # the torus mixes x without the RMSNorm
                    out[f"l{l}_g{nm}"] = gn.numpy()
        if cfg.get("active"):
            gv = [c.V.weight.grad for c in layer.christoffels if getattr(c, "V", None) is not None]
            if gv and gv[0] is not None:
                out[f"l{l}_V"] = np.stack([t.numpy() for t in gv])
            g0 = layer.gatings[0].curvature_net[0].weight.grad
            if g0 is not None:
                out[f"l{l}_gate_W1"] = np.stack([g.curvature_net[0].weight.grad.numpy() for g in layer.gatings])
                out[f"l{l}_gate_b2"] = np.stack([g.curvature_net[2].bias.grad.numpy() for g in layer.gatings])
            if getattr(layer, "context_proj", None) is not None and layer.context_proj.weight.grad is not None:
                out[f"l{l}_ctx_W"] = layer.context_proj.weight.grad.numpy()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(name, len(out))


INIT_CONFIGS = {
    "c1_init": dict(vocab_size=2, dim=128, depth=4, rank=16, heads=4, integrator_type="leapfrog",
                    base_dt=0.1),
    "func_init": dict(vocab_size=300, dim=64, depth=2, rank=16, heads=4, integrator_type="leapfrog",
                      base_dt=0.1, physics_config={"embedding": {"type": "functional"}}),
    "scan_init": dict(vocab_size=50, dim=32, depth=2, heads=4, integrator_type="leapfrog",
                      use_scan=True),
    "heun_init": dict(vocab_size=9, dim=32, depth=2, rank=8, heads=2, base_dt=0.1),
    "torus_init": dict(vocab_size=9, dim=32, depth=2, rank=8, heads=2, integrator_type="rk4", base_dt=0.1,
                       physics_config={"topology": {"type": "torus"}}),
}


def gen_init():
    """Checksums of the reference's own initial weights under torch.manual_seed(3):
    the drop-in model must reproduce them exactly (same modules, same init order)."""
    import json
    out = {}
    for name, kw in INIT_CONFIGS.items():
        torch.manual_seed(3)
        with contextlib.redirect_stdout(io.StringIO()):
            m = Manifold(**kw)
        sd = m.state_dict()
        out[name] = {k: [float(v.double().sum()), float(v.double().abs().sum()),
                         [float(t) for t in v.reshape(-1)[:3].double()]] for k, v in sd.items()}
    with open(os.path.join(HERE, "init_checksums.json"), "w") as fh:
        json.dump(dict(configs={k: {kk: vv for kk, vv in v.items() if kk != "physics_config"}
                                for k, v in INIT_CONFIGS.items()},
                       physics={k: v.get("physics_config") for k, v in INIT_CONFIGS.items()},
                       sums=out), fh)
    print("init", {k: len(v) for k, v in out.items()})


if __name__ == "__main__":
    names = sys.argv[1:] or list(C.CASES)
    for n in names:
        if n == "units":
            gen_units()
        elif n == "ops":
            gen_ops()
        elif n == "init":
            gen_init()
        elif n in C.GRAD_CASES:
            gen_grad_case(n, C.GRAD_CASES[n])
        elif n in C.GENERIC_GRAD_CASES:
            gen_grad_case(n, C.GENERIC_GRAD_CASES[n])
        else:
            gen_model_case(n, C.CASES[n])
    if not sys.argv[1:]:
        gen_units()
        gen_ops()
        gen_init()
        for n, cfg in C.GRAD_CASES.items():
            gen_grad_case(n, cfg)
