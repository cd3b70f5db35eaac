"""Host-side checks that need no GPU: the C-ABI library loads and exports
every declared symbol, the layout arithmetic, the drop-in module tree and
initialisation, and that nothing runs on CPU tensors (no CPU fallback)."""
import json
import os
import re

import pytest
import torch

import manifold_b200 as gfn
from manifold_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "gfn_b200.h")).read()
    return sorted(set(re.findall(r"\b(gfn_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/gfn_b200.h but not exported"
    assert set(syms) == set(_lib.EXPORTED), "ctypes signature table out of sync with the header"
    assert b"sm_100a" in lib.gfn_build_info()


def test_status_strings():
    lib = _lib.load()
    assert lib.gfn_status_string(0) == b"ok"
    assert lib.gfn_status_string(2) == b"unsupported configuration"


def test_pack_layout_sizes():
    lib = _lib.load()
    # d=256, H=8 -> cluster 8, 32 columns per CTA, k-chunk 64: 4 chunks of
    # 64 rows x (64 + 4 pad) floats, after a head section of
    # WfT 32x32 | U, W 32x4 | bf, bx, bv, gx, gv 5x32 | softplus(dt) 1, padded to 32
    head = 32 * 32 + 2 * 32 * 4 + 5 * 32
    head = (head + 1 + 31) // 32 * 32
    assert lib.gfn_leapfrog_pack_floats(256, 8, 4, 6) == 6 * 8 * (head + 4 * 64 * 68)
    assert lib.gfn_leapfrog_pack_floats(256, 8, 5, 6) == -1   # rank 5 unsupported
    assert lib.gfn_leapfrog_pack_floats(250, 8, 4, 6) == -1   # heads must divide dim
    assert lib.gfn_leapfrog_pack_floats(16, 1, 4, 2) > 0      # single head: no mixing


def test_invalid_arguments_are_rejected_before_launch():
    lib = _lib.load()
    st = lib.gfn_leapfrog_pack(None, None, None, None, None, None, None, None, None, None, None,
                               256, 8, 4, 6, None, 0, None)
    assert st == 1
    assert b"NULL" in lib.gfn_last_error_message()
    assert lib.gfn_parallel_scan(None, None, None, None, 0, 1, 1, 4, None) == 1


def test_init_matches_reference_checksums():
    """Same seed -> same initial weights as the reference (module tree and
    init order mirrored); checksums recorded from the reference itself."""
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "init_checksums.json")))
    for name, kw in g["configs"].items():
        kw = dict(kw)
        if g["physics"].get(name):
            kw["physics_config"] = g["physics"][name]
        torch.manual_seed(3)
        m = gfn.Manifold(**kw)
        sd = m.state_dict()
        ref = g["sums"][name]
        assert set(sd) == set(ref), name
        for k, (s, sa, head) in ref.items():
            v = sd[k].double()
            assert abs(float(v.sum()) - s) <= 1e-9 * max(1.0, abs(sa)), (name, k)
            assert [float(t) for t in v.reshape(-1)[:3]] == head, (name, k)


def test_unsupported_configurations_raise():
    for integ in ("coupling", "neural"):
        with pytest.raises(gfn.GfnError):
            gfn.Manifold(vocab_size=4, dim=32, depth=1, heads=2, integrator_type=integ)
    with pytest.raises(gfn.GfnError):
        gfn.Manifold(vocab_size=4, dim=32, depth=1, heads=2, integrator_type="leapfrog",
                     physics_config={"mixture": {"enabled": True}})
    # the torus and the other integrators build (generic path)
    m = gfn.Manifold(vocab_size=4, dim=32, depth=1, heads=2, integrator_type="heun",
                     physics_config={"topology": {"type": "torus"}})
    assert m.layers[0].generic and m.layers[0].out_proj_x.in_features == 96


def test_no_cpu_fallback():
    m = gfn.Manifold(vocab_size=4, dim=32, depth=1, heads=2, integrator_type="leapfrog")
    ids = torch.zeros(1, 3, dtype=torch.long)
    with pytest.raises(gfn.GfnError):
        with torch.no_grad():
            m(ids)
    with pytest.raises(gfn.GfnError):
        gfn.parallel_scan(torch.ones(1, 4, 4), torch.ones(1, 4, 4))
    with pytest.raises(gfn.GfnError):
        m.layers[0](torch.zeros(1, 32), torch.zeros(1, 32), torch.zeros(1, 32))


def test_cross_entropy_loss_host_checks():
    import manifold_b200 as gfn
    with pytest.raises(gfn.GfnError):
        gfn.CrossEntropyLoss(label_smoothing=0.1)
    with pytest.raises(gfn.GfnError):
        gfn.CrossEntropyLoss(weight=torch.ones(3))
    with pytest.raises(gfn.GfnError):  # no CPU path
        gfn.cross_entropy(torch.zeros(2, 3), torch.zeros(2, dtype=torch.int64))


def test_training_routing_by_head_dim():
    # the fused BPTT kernels take head_dim <= 64; larger heads (and the generic
    # configurations) train through the generic layer step
    import manifold_b200 as gfn
    small = gfn.Manifold(vocab_size=7, dim=64, depth=1, rank=8, heads=1, integrator_type="leapfrog")
    big = gfn.Manifold(vocab_size=7, dim=256, depth=1, rank=8, heads=2, integrator_type="leapfrog")
    heun = gfn.Manifold(vocab_size=7, dim=64, depth=1, rank=8, heads=2, integrator_type="heun")
    assert not small.layers[0].training_generic()
    assert big.layers[0].training_generic() and not big.layers[0].generic
    assert heun.layers[0].training_generic() and heun.layers[0].generic
