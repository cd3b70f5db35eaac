"""CUDA path vs the reference (golden fixtures) and vs the numpy oracle.

All calls go through manifold_b200's Python API, which calls the C ABI of
libgfn_b200.so.  Tolerances:
  - per layer step (teacher forced, identical input state): rowwise
    |a - b| <= 1e-6 + 1e-5 * max|b_row|   (tests/parity.py)
  - free-running sequences: the same form with rtol 1e-4, atol 1e-5, since
    float32 rounding differences compound over tokens x layers
  - bfloat16 forces (the LM-prefill variant) vs the float32 reference:
    rtol 2e-2 (bfloat16 keeps 8 mantissa bits)
"""
import os

import numpy as np
import pytest
import torch

from oracle import gfn_oracle as O
from tests.golden import cases as C
from tests.parity import max_rel, report, rowwise_close

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
SEQ_RTOL, SEQ_ATOL = 1e-4, 1e-5


def load(name):
    return dict(np.load(os.path.join(GOLD, f"{name}.npz")))


def build(cfg, P=None):
    import manifold_b200 as gfn
    torch.manual_seed(0)
    m = gfn.Manifold(**C.model_kwargs(cfg)).cuda().eval()
    C.load_into_model(m, cfg, P if P is not None else C.make_params(cfg))
    return m


def cu(a):
    return torch.as_tensor(np.asarray(a)).cuda()


@pytest.mark.parametrize("name", ["tiny", "h1", "mask", "c1", "c2s", "c3s", "c4s", "c5s"])
def test_sequence_matches_reference(name):
    cfg = C.CASES[name]
    g = load(name)
    m = build(cfg)
    mask = cu(g["mask"]) if "mask" in g else None
    with torch.no_grad():
        x_seq, v_seq, (x, v), _ = m.recurrence(cu(g["ids"]), attention_mask=mask)
    rowwise_close(x_seq.cpu().numpy(), g["x_seq"], SEQ_RTOL, SEQ_ATOL, "x_seq")
    rowwise_close(v_seq.cpu().numpy(), g["v_seq"], SEQ_RTOL, SEQ_ATOL, "v_seq")
    rowwise_close(x.cpu().numpy(), g["x_final"], SEQ_RTOL, SEQ_ATOL, "x_final")
    rowwise_close(v.cpu().numpy(), g["v_final"], SEQ_RTOL, SEQ_ATOL, "v_final")


def test_forward_api_returns_reference_tuple():
    cfg = C.CASES["tiny"]
    g = load("tiny")
    m = build(cfg)
    with torch.no_grad():
        out = m(cu(g["ids"]))
    assert len(out) == 6
    logits, (x, v), christ, v_seq, x_seq, forces = out
    assert logits.shape == (cfg["B"], cfg["L"], cfg["V"])
    assert len(x_seq) == cfg["L"] and x_seq[0].shape == (cfg["B"], cfg["d"])
    rowwise_close(torch.stack(x_seq, 1).cpu().numpy(), g["x_seq"], SEQ_RTOL, SEQ_ATOL, "x_seq")
    np.testing.assert_allclose(forces.cpu().numpy(), C.make_params(cfg)["emb"][g["ids"]])


@pytest.mark.parametrize("name", ["c2s", "c3s", "c4s"])
def test_layer_step_matches_reference(name):
    """Teacher-forced single MLayer step (per-step parity bar)."""
    cfg = C.CASES[name]
    g = load(name)
    m = build(cfg)
    layer = m.layers[int(g["step_layer"])]
    layer.recurrence_path = "fused"
    with torch.no_grad():
        xo, vo, ctx, _ = layer(cu(g["step_x"]), cu(g["step_v"]), cu(g["step_F"]))
    report(xo.cpu().numpy(), g["step_xo"], f"{name} fused step x")
    report(vo.cpu().numpy(), g["step_vo"], f"{name} fused step v")
    rowwise_close(xo.cpu().numpy(), g["step_xo"], what="x")
    rowwise_close(vo.cpu().numpy(), g["step_vo"], what="v")
    assert ctx.shape == (5, cfg["H"])


@pytest.mark.parametrize("name", ["c3s", "c4s"])
def test_layer_step_layered_matches_reference(name, mixing):
    """Teacher-forced single MLayer step through the layered (large batch)
    path, in every mixing arithmetic, at the per-step bar."""
    cfg = C.CASES[name]
    g = load(name)
    m = build(cfg)
    layer = m.layers[int(g["step_layer"])]
    layer.recurrence_path = "layered"
    with torch.no_grad():
        xo, vo, _, _ = layer(cu(g["step_x"]), cu(g["step_v"]), cu(g["step_F"]))
    report(xo.cpu().numpy(), g["step_xo"], f"{name} layered/{mixing} step x")
    report(vo.cpu().numpy(), g["step_vo"], f"{name} layered/{mixing} step v")
    rowwise_close(xo.cpu().numpy(), g["step_xo"], what="x")
    rowwise_close(vo.cpu().numpy(), g["step_vo"], what="v")


def test_c4_layer_step_full_batch_layered(mixing):
    """C4 layer shape at the full decode batch (4096 rows), teacher forced:
    one layered layer step from random states vs the float64 oracle on 48
    sampled rows, at the per-step bar."""
    cfg = dict(C.CASES["c4s"], B=4096, L=1, seed=9)
    P = C.make_params(cfg)
    m = build(cfg, P)
    li = 5
    layer = m.layers[li]
    layer.recurrence_path = "layered"
    d = cfg["d"]
    rng = np.random.default_rng(11)
    x = rng.standard_normal((4096, d)).astype(np.float32)
    v = (rng.standard_normal((4096, d)) * 2).astype(np.float32)
    F = P["emb"][rng.integers(0, cfg["V"], 4096)]
    with torch.no_grad():
        xo, vo, _, _ = layer(cu(x), cu(v), cu(F))
    rows = np.r_[0:16, 2040:2056, 4080:4096]
    lp = {k: a.astype(np.float64) for k, a in P["layers"][li].items()}
    ox, ov = O.mlayer_step(x[rows].astype(np.float64), v[rows].astype(np.float64),
                           F[rows].astype(np.float64), lp, cfg["H"], cfg["dt"])
    xo, vo = xo.cpu().numpy()[rows], vo.cpu().numpy()[rows]
    report(xo, ox, f"C4 full-batch layered/{mixing} step x vs float64")
    report(vo, ov, f"C4 full-batch layered/{mixing} step v vs float64")
    rowwise_close(xo, ox, what="x")
    rowwise_close(vo, ov, what="v")


def test_decode_streaming_state_c4s():
    """Batched decode: one token per call with the (x, v) state carried."""
    cfg = C.CASES["c4s"]
    g = load("c4s")
    m = build(cfg)
    with torch.no_grad():
        _, _, st, _ = m.recurrence(cu(g["ids"]))
        _, _, (x2, v2), _ = m.recurrence(cu(g["ids2"]), state=st)
    rowwise_close(x2.cpu().numpy(), g["x_final2"], SEQ_RTOL, SEQ_ATOL, "x")
    rowwise_close(v2.cpu().numpy(), g["v_final2"], SEQ_RTOL, SEQ_ATOL, "v")


def test_functional_embedding_matches_reference():
    cfg = C.CASES["c3s"]
    g = load("c3s")
    m = build(cfg)
    with torch.no_grad():
        f32 = m.embedding(cu(g["ids"]))
        bf = m.embedding(cu(g["ids"]), out_dtype=torch.bfloat16)
    np.testing.assert_allclose(f32.cpu().numpy(), g["forces"], rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(bf.float().cpu().numpy(), g["forces"], rtol=2 ** -8, atol=1e-6)


def test_bf16_forces_variant():
    """bf16 forces / fp32 state (the LM-prefill variant) vs the fp32 reference."""
    cfg = C.CASES["c3s"]
    g = load("c3s")
    m = build(cfg)
    m.force_dtype = torch.bfloat16
    with torch.no_grad():
        x_seq, _, _, forces = m.recurrence(cu(g["ids"]))
    assert forces.dtype == torch.bfloat16
    err = max_rel(x_seq.cpu().numpy(), g["x_seq"])
    print(f"bf16-force variant: max rowwise relative error vs fp32 reference = {err:.3e}")
    rowwise_close(x_seq.cpu().numpy(), g["x_seq"], 2e-2, 1e-4, "x_seq(bf16 forces)")


def test_units_match_reference():
    from manifold_b200.cuda import ops
    g = load("units")
    gam = ops.christoffel_fused(cu(g["ch_v"]), cu(g["ch_U"]), cu(g["ch_W"]))
    rowwise_close(gam.cpu().numpy(), g["ch_gamma"], what="gamma")
    xn, vn = ops.leapfrog_fused(cu(g["lf_x"]), cu(g["ch_v"]), cu(g["lf_F"]), cu(g["ch_U"]),
                                cu(g["ch_W"]), 0.1, torch.tensor([0.87]).cuda(), 3,
                                Wf=cu(g["lf_Wf"]), bf=cu(g["lf_bf"]))
    rowwise_close(xn.detach().cpu().numpy(), g["lf_xn"], what="x")
    rowwise_close(vn.detach().cpu().numpy(), g["lf_vn"], what="v")
    for L in (20, 100):
        y = ops.parallel_scan_fused(cu(g[f"scan{L}_a"]), cu(g[f"scan{L}_x"]))
        rowwise_close(y.cpu().numpy(), g[f"scan{L}_y"], 1e-5, 1e-6, f"scan{L}")


def test_integrator_module_matches_reference():
    import manifold_b200 as gfn
    g = load("units")
    ch = gfn.LowRankChristoffel(24, 4).cuda()
    with torch.no_grad():
        ch.U.copy_(cu(g["ch_U"]))
        ch.W.copy_(cu(g["ch_W"]))
    integ = gfn.LeapfrogIntegrator(ch, dt=0.1)
    xn, vn = integ(cu(g["lf_x"]), cu(g["ch_v"]), force=cu(g["lf_F"]),
                   dt_scale=torch.tensor([[0.87]]).cuda(), steps=3,
                   W_forget_stack=cu(g["lf_Wf"])[None], b_forget_stack=cu(g["lf_bf"])[None])
    rowwise_close(xn.detach().cpu().numpy(), g["lf_xn"], what="x")
    rowwise_close(vn.detach().cpu().numpy(), g["lf_vn"], what="v")


def test_parallel_layer_matches_reference():
    import manifold_b200 as gfn
    g = load("units")
    pl = gfn.ParallelMLayer(32, heads=4).cuda()
    with torch.no_grad():
        pl.norm_x.weight.copy_(cu(g["pl_ln_w"])); pl.norm_x.bias.copy_(cu(g["pl_ln_b"]))
        pl.to_A[0].weight.copy_(cu(g["pl_WA"])); pl.to_A[0].bias.copy_(cu(g["pl_bA"]))
        pl.to_dt[0].weight.copy_(cu(g["pl_Wdt"])); pl.to_dt[0].bias.copy_(cu(g["pl_bdt"]))
        pl.to_B.weight.copy_(cu(g["pl_WB"])); pl.to_B.bias.copy_(cu(g["pl_bB"]))
        xs, vs, _, _ = pl(None, None, cu(g["pl_f"]))
    rowwise_close(xs.cpu().numpy(), g["pl_x"], 1e-4, 1e-5, "x_seq")
    rowwise_close(vs.cpu().numpy(), g["pl_v"], 1e-4, 1e-5, "v_seq")


# ---------------------------------------------------------------- full sizes
def _big(cfg_name, B, L, seed=5):
    cfg = dict(C.CASES[cfg_name], B=B, L=L, seed=seed)
    P = C.make_params(cfg)
    ids = np.random.default_rng(seed).integers(0, cfg["V"], (B, L)).astype(np.int64)
    return cfg, P, ids


def test_c2_full_batch_vs_oracle_and_streaming_is_exact():
    """C2 shapes (d=256, 6 layers, 8 heads, B=64): oracle parity over a short
    slice, bitwise determinism, and chunked streaming == one call (bitwise)."""
    cfg, P, ids = _big("c2s", 64, 16)
    m = build(cfg, P)
    idt = cu(ids)
    with torch.no_grad():
        xs, vs, (x, v), _ = m.recurrence(idt)
        xs2, _, _, _ = m.recurrence(idt)
        a, _, st, _ = m.recurrence(idt[:, :7])
        b, _, (xb, vb), _ = m.recurrence(idt[:, 7:], state=st)
    assert torch.equal(xs, xs2), "not deterministic"
    assert torch.equal(torch.cat([a, b], 1), xs), "streamed chunks differ from one call"
    assert torch.equal(xb, x) and torch.equal(vb, v)
    F = P["emb"][ids]
    x0 = np.broadcast_to(P["x0"], (64, cfg["d"])).copy()
    v0 = np.broadcast_to(P["v0"], (64, cfg["d"])).copy()
    oxs, ovs, _, _ = O.manifold_forward(x0, v0, F[:, :4], P["layers"], cfg["H"], cfg["dt"])
    rowwise_close(xs[:, :4].cpu().numpy(), oxs, SEQ_RTOL, SEQ_ATOL, "x_seq")
    rowwise_close(vs[:, :4].cpu().numpy(), ovs, SEQ_RTOL, SEQ_ATOL, "v_seq")


def test_c4_full_decode_step_vs_oracle():
    """C4: B=4096 streams, d=1024, 24 layers, 16 heads, one decode step.
    Rows are independent; 48 of them are checked against the oracle."""
    cfg, P, ids = _big("c4s", 4096, 1)
    m = build(cfg, P)
    rng = np.random.default_rng(7)
    x0 = rng.standard_normal((4096, cfg["d"])).astype(np.float32)
    v0 = (rng.standard_normal((4096, cfg["d"])) * 2).astype(np.float32)
    with torch.no_grad():
        _, _, (x, v), _ = m.recurrence(cu(ids), state=(cu(x0), cu(v0)))
    rows = np.r_[0:16, 2040:2056, 4080:4096]
    F = P["emb"][ids[rows]]
    _, _, ox, ov = O.manifold_forward(x0[rows], v0[rows], F, P["layers"], cfg["H"], cfg["dt"])
    rowwise_close(x.cpu().numpy()[rows], ox, SEQ_RTOL, SEQ_ATOL, "x")
    rowwise_close(v.cpu().numpy()[rows], ov, SEQ_RTOL, SEQ_ATOL, "v")


def test_c3_shapes_full_batch_slice_vs_oracle():
    """C3 shapes (d=512, 12 layers, 8 heads) at the full batch 256, 2 tokens."""
    cfg = dict(C.CASES["c3s"], B=256, L=2, seed=21)
    P = C.make_params(cfg)
    ids = C.zipf_ids(np.random.default_rng(3), cfg["V"], (256, 2))
    m = build(cfg, P)
    with torch.no_grad():
        xs, _, _, forces = m.recurrence(cu(ids))
    F = O.functional_embedding(ids, P["func"])
    np.testing.assert_allclose(forces.cpu().numpy(), F, rtol=1e-5, atol=2e-6)
    rows = np.r_[0:8, 250:256]
    x0 = np.broadcast_to(P["x0"], (len(rows), cfg["d"])).copy()
    v0 = np.broadcast_to(P["v0"], (len(rows), cfg["d"])).copy()
    oxs, _, _, _ = O.manifold_forward(x0, v0, F[rows], P["layers"], cfg["H"], cfg["dt"])
    rowwise_close(xs.cpu().numpy()[rows], oxs, SEQ_RTOL, SEQ_ATOL, "x_seq")


def test_c3_full_batch_64_tokens_vs_oracle():
    """C3 shapes at the full batch 256 over 64 tokens (layered path, bf16
    functional forces as in the LM-prefill config): 6 sampled rows against
    the oracle fed the same bf16-rounded forces, free-running bar."""
    cfg = dict(C.CASES["c3s"], B=256, L=64, seed=23)
    P = C.make_params(cfg)
    ids = C.zipf_ids(np.random.default_rng(4), cfg["V"], (256, 64))
    m = build(cfg, P)
    m.force_dtype = torch.bfloat16
    assert m._use_layered(256)
    with torch.no_grad():
        xs, vs, (x, v), forces = m.recurrence(cu(ids))
    rows = np.r_[0:3, 253:256]
    F = forces.float().cpu().numpy()[rows]
    x0 = np.broadcast_to(P["x0"], (len(rows), cfg["d"])).copy()
    v0 = np.broadcast_to(P["v0"], (len(rows), cfg["d"])).copy()
    oxs, ovs, _, _ = O.manifold_forward(x0, v0, F, P["layers"], cfg["H"], cfg["dt"])
    report(xs.cpu().numpy()[rows], oxs, "C3 64 tokens x_seq")
    rowwise_close(xs.cpu().numpy()[rows], oxs, SEQ_RTOL, SEQ_ATOL, "x_seq")
    rowwise_close(vs.cpu().numpy()[rows], ovs, SEQ_RTOL, SEQ_ATOL, "v_seq")


def test_scan_long_and_chunked_paths():
    from manifold_b200.cuda import ops
    rng = np.random.default_rng(1)
    for B, L, D in ((2, 4096, 8), (4, 777, 64), (3, 33, 4)):
        a = rng.uniform(0.8, 1.0, (B, L, D)).astype(np.float32)
        x = rng.standard_normal((B, L, D)).astype(np.float32)
        ref = O.scan_sequential(a.astype(np.float64), x.astype(np.float64))
        for ws in (True, False):
            y = ops.parallel_scan_fused(cu(a), cu(x), workspace=ws).cpu().numpy()
            rowwise_close(y, ref, 1e-5, 1e-5, f"scan {B}x{L}x{D} ws={ws}")
        y1 = ops.parallel_scan_fused(None, cu(x)).cpu().numpy()
        rowwise_close(y1, np.cumsum(x.astype(np.float64), 1), 1e-5, 1e-4, "cumsum")


def test_scan_path_model_matches_oracle():
    import manifold_b200 as gfn
    torch.manual_seed(0)
    m = gfn.Manifold(vocab_size=50, dim=64, depth=3, heads=4, integrator_type="leapfrog",
                     use_scan=True).cuda().eval()
    ids = torch.randint(0, 50, (4, 70)).cuda()
    with torch.no_grad():
        logits, (xl, _), _ = m(ids)
        f = m.embedding(ids)
    cur = f.cpu().numpy()
    for layer in m.layers:
        pp = dict(ln_w=layer.norm_x.weight, ln_b=layer.norm_x.bias, WA=layer.to_A[0].weight,
                  bA=layer.to_A[0].bias, Wdt=layer.to_dt[0].weight, bdt=layer.to_dt[0].bias,
                  WB=layer.to_B.weight, bB=layer.to_B.bias)
        pp = {k: t.detach().cpu().numpy() for k, t in pp.items()}
        cur, _ = O.parallel_mlayer(cur, pp, 4)
    xn = O.layernorm(cur, m.readout_norm.weight.detach().cpu().numpy(),
                     m.readout_norm.bias.detach().cpu().numpy())
    rowwise_close(xl.cpu().numpy(), xn[:, -1], 1e-4, 1e-5, "x_final")


# ---------------------------------------------------------------- errors
def test_errors_are_loud():
    import manifold_b200 as gfn
    from manifold_b200.cuda import ops
    cfg = C.CASES["tiny"]
    m = build(cfg)
    with pytest.raises(gfn.GfnError):
        ops.christoffel_fused(torch.zeros(2, 8), torch.zeros(8, 4), torch.zeros(8, 4))  # CPU
    with pytest.raises(gfn.GfnError):
        ops.christoffel_fused(torch.zeros(2, 8).cuda(), torch.zeros(8, 5).cuda(), torch.zeros(8, 5).cuda())
    ops.device_error(reset=True)
    bad = torch.tensor([[0, 1, 99]], device="cuda")
    with torch.no_grad():
        m.recurrence(bad)
    assert ops.device_error(reset=True) & 2, "out-of-range token id not reported"
    assert ops.device_error(reset=True) == 0


@pytest.fixture(params=["umma_f16", "umma_f16+tc_head", "split_bf16", "fp32_simt", "split_f16"])
def mixing(request):
    """Mixing arithmetic of the layered path; "+tc_head" also forces the
    tensor-core head-step kernel (head_dim 64) at any batch size."""
    from manifold_b200.cuda import ops
    name = request.param.split("+")[0]
    mode = {"split_bf16": ops.MIX_SPLIT_BF16, "fp32_simt": ops.MIX_FP32_SIMT,
            "split_f16": ops.MIX_SPLIT_F16, "umma_f16": ops.MIX_UMMA_F16}[name]
    prev = ops.set_layered_mixing(mode)
    old = os.environ.get("GFN_LAY_HEAD")
    os.environ["GFN_LAY_HEAD"] = "1" if "tc_head" in request.param else "0"
    yield request.param
    ops.set_layered_mixing(prev)
    if old is None:
        del os.environ["GFN_LAY_HEAD"]
    else:
        os.environ["GFN_LAY_HEAD"] = old


@pytest.mark.parametrize("name", ["tiny", "mask", "c1", "c2s", "c3s", "c4s", "c5s"])
def test_layered_sequence_matches_reference(name, mixing):
    """The layer-by-layer (large batch) path against the same goldens, with
    either mixing-GEMM arithmetic."""
    cfg = C.CASES[name]
    if cfg["H"] == 1:
        pytest.skip("layered path needs head mixing")
    g = load(name)
    m = build(cfg)
    m.recurrence_path = "layered"
    mask = cu(g["mask"]) if "mask" in g else None
    with torch.no_grad():
        x_seq, v_seq, (x, v), _ = m.recurrence(cu(g["ids"]), attention_mask=mask)
    rowwise_close(x_seq.cpu().numpy(), g["x_seq"], SEQ_RTOL, SEQ_ATOL, "x_seq")
    rowwise_close(v_seq.cpu().numpy(), g["v_seq"], SEQ_RTOL, SEQ_ATOL, "v_seq")
    rowwise_close(x.cpu().numpy(), g["x_final"], SEQ_RTOL, SEQ_ATOL, "x_final")
    rowwise_close(v.cpu().numpy(), g["v_final"], SEQ_RTOL, SEQ_ATOL, "v_final")


def test_layered_matches_fused_c4_shape(mixing):
    """C4 layer shape (d=1024, 16 heads, rank 64) at a batch of 512 with a
    carried state: layered and fused paths agree, and both continue a
    split sequence exactly like the unsplit one."""
    import manifold_b200 as gfn
    torch.manual_seed(0)
    m = gfn.Manifold(vocab_size=1000, dim=1024, depth=2, rank=64, heads=16,
                     integrator_type="leapfrog").cuda().eval()
    ids = torch.randint(0, 1000, (512, 4), device="cuda")
    with torch.no_grad():
        m.recurrence_path = "fused"
        xf_seq, vf_seq, (xf, vf), _ = m.recurrence(ids)
        m.recurrence_path = "layered"
        xl_seq, vl_seq, (xl, vl), _ = m.recurrence(ids)
        _, _, st, _ = m.recurrence(ids[:, :2])
        xs2, _, (x2, v2), _ = m.recurrence(ids[:, 2:], state=st)
    rowwise_close(xl_seq.cpu().numpy(), xf_seq.cpu().numpy(), SEQ_RTOL, SEQ_ATOL, "x_seq")
    rowwise_close(vl_seq.cpu().numpy(), vf_seq.cpu().numpy(), SEQ_RTOL, SEQ_ATOL, "v_seq")
    torch.testing.assert_close(xs2, xl_seq[:, 2:], rtol=0, atol=0)
    torch.testing.assert_close(x2, xl, rtol=0, atol=0)
    torch.testing.assert_close(v2, vl, rtol=0, atol=0)


@pytest.mark.parametrize("d,H,rank,B", [(256, 4, 32, 100), (256, 4, 64, 70), (256, 2, 8, 33),
                                        (512, 16, 64, 129), (128, 8, 128, 65)])
def test_layered_matches_fused_shapes(d, H, rank, B, mixing):
    """Head dims 16-128 and per-head ranks 4-16 on ragged row tiles, bf16
    forces: the layered path agrees with the fused kernel."""
    import manifold_b200 as gfn
    torch.manual_seed(1)
    m = gfn.Manifold(vocab_size=50, dim=d, depth=2, rank=rank, heads=H,
                     integrator_type="leapfrog").cuda().eval()
    with torch.no_grad():
        for layer in m.layers:
            for ch in layer.christoffels:
                ch.U.normal_(0, 0.1)
                ch.W.normal_(0, 0.1)
    F = (torch.randn(B, 3, d, device="cuda") * 0.5).to(torch.bfloat16)
    with torch.no_grad():
        m.recurrence_path = "fused"
        xf, vf, _, _ = m.recurrence(force_manual=F)
        m.recurrence_path = "layered"
        xl, vl, _, _ = m.recurrence(force_manual=F)
    rowwise_close(xl.cpu().numpy(), xf.cpu().numpy(), SEQ_RTOL, SEQ_ATOL, "x_seq")
    rowwise_close(vl.cpu().numpy(), vf.cpu().numpy(), SEQ_RTOL, SEQ_ATOL, "v_seq")


def test_layered_f16_range_flag():
    """Activations beyond the split-fp16 range are reported through the device
    error word (no fault); the bf16 split handles the same input."""
    import manifold_b200 as gfn
    from manifold_b200 import _lib
    from manifold_b200.cuda import ops
    torch.manual_seed(2)
    m = gfn.Manifold(vocab_size=10, dim=256, depth=1, rank=32, heads=4,
                     integrator_type="leapfrog").cuda().eval()
    m.recurrence_path = "layered"
    F = torch.full((8, 1, 256), 2.0e6, device="cuda")
    _lib.device_error(reset=True)
    prev = ops.set_layered_mixing(ops.MIX_SPLIT_F16)
    try:
        with torch.no_grad():
            m.recurrence(force_manual=F)
        torch.cuda.synchronize()
        assert _lib.device_error(reset=True) & 4
        ops.set_layered_mixing(ops.MIX_SPLIT_BF16)
        with torch.no_grad():
            x, v, _, _ = m.recurrence(force_manual=F)
        torch.cuda.synchronize()
        assert _lib.device_error(reset=True) & 4 == 0
        assert torch.isfinite(x).all() and torch.isfinite(v).all()
    finally:
        ops.set_layered_mixing(prev)
