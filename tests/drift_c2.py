"""Long-horizon drift of the C2 recurrence (d=256, 6 layers, 8 heads, rank 32,
batch 64, parity-bit tokens) over 100k tokens.

Test infrastructure, not part of the product; two phases:

  python tests/drift_c2.py gpu --out DRIFT.npz
      (B200) streams the whole batch through Manifold.recurrence in 2000-token
      chunks with the state carried between calls and records rows 0..R-1 of
      (x, v) every `--every` tokens.
  python tests/drift_c2.py cpu --gpu DRIFT.npz
      (host) replays the same rows with the numpy oracle (the reference's
      algorithm, oracle/gfn_oracle.py) in float64 and float32 and prints, per
      checkpoint, the row-relative L2 distance of the GPU state and of the
      float32 oracle state from the float64 oracle state.

Weights are the seeded C2 parameters of tests/golden/cases.py; tokens are
seeded Bernoulli(0.5) bits (the synthetic stand-in for the reference's parity
task).
"""
import argparse
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from tests.golden import cases as C  # noqa: E402

CFG = dict(V=2, d=256, NL=6, H=8, rank=32, B=64, dt=0.1, seed=2024)


def tokens(n, B):
    rng = np.random.default_rng(77)
    return rng.integers(0, 2, size=(B, n), dtype=np.int64)


def run_gpu(args):
    import torch
    import manifold_b200 as gfn
    P = C.make_params(CFG)
    torch.manual_seed(0)
    m = gfn.Manifold(**C.model_kwargs(CFG)).cuda().eval()
    C.load_into_model(m, CFG, P)
    ids = tokens(args.tokens, CFG["B"])
    chunk, every, R = 2000, args.every, args.rows
    assert chunk % every == 0
    xs, vs = [], []
    st = None
    t0 = time.time()
    with torch.no_grad():
        for s in range(0, args.tokens, chunk):
            idc = torch.from_numpy(ids[:, s:s + chunk]).cuda()
            x_seq, v_seq, st, _ = m.recurrence(idc, state=st)
            sel = slice(every - 1, chunk, every)
            xs.append(x_seq[:R, sel].cpu().numpy())
            vs.append(v_seq[:R, sel].cpu().numpy())
    torch.cuda.synchronize()
    print(f"gpu: {args.tokens} tokens x {CFG['B']} rows in {time.time() - t0:.1f} s")
    np.savez_compressed(args.out, x=np.concatenate(xs, 1), v=np.concatenate(vs, 1),
                        every=every, tokens=args.tokens, rows=R)


def run_cpu(args):
    from oracle import gfn_oracle as O
    g = np.load(args.gpu)
    every, n, R = int(g["every"]), int(g["tokens"]), int(g["rows"])
    P = C.make_params(CFG)
    ids = tokens(n, CFG["B"])[:R]
    out = {}
    for dt in (np.float64, np.float32):
        layers = [{k: (v.astype(dt) if isinstance(v, np.ndarray) else v) for k, v in lp.items()}
                  for lp in P["layers"]]
        emb = P["emb"].astype(dt)
        x = np.broadcast_to(P["x0"].astype(dt), (R, CFG["d"])).copy()
        v = np.broadcast_to(P["v0"].astype(dt), (R, CFG["d"])).copy()
        xs, vs = [], []
        t0 = time.time()
        for s in range(0, n, every):
            F = emb[ids[:, s:s + every]]
            _, _, x, v = O.manifold_forward(x, v, F, layers, CFG["H"], CFG["dt"])
            xs.append(x.copy())
            vs.append(v.copy())
        out[dt] = (np.stack(xs, 1), np.stack(vs, 1))
        print(f"oracle {np.dtype(dt).name}: {time.time() - t0:.0f} s", flush=True)

    def rel(a, b):  # [R, K, d] -> max over rows of the row-relative L2 distance, per checkpoint
        num = np.linalg.norm(a.astype(np.float64) - b, axis=-1)
        den = np.linalg.norm(b, axis=-1) + 1e-30
        return (num / den).max(0)

    x64, v64 = out[np.float64]
    x32, v32 = out[np.float32]
    gx = rel(g["x"], x64)
    gv = rel(g["v"], v64)
    ox = rel(x32, x64)
    ov = rel(v32, v64)
    print("| tokens | GPU x vs fp64 | GPU v vs fp64 | oracle fp32 x vs fp64 | oracle fp32 v vs fp64 |")
    print("|---|---|---|---|---|")
    K = gx.shape[0]
    for k in sorted(set([0, 1, 4, 9, 24, 49, 99, K - 1]) & set(range(K))):
        print(f"| {(k + 1) * every} | {gx[k]:.2e} | {gv[k]:.2e} | {ox[k]:.2e} | {ov[k]:.2e} |")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("phase", choices=["gpu", "cpu"])
    ap.add_argument("--tokens", type=int, default=100000)
    ap.add_argument("--every", type=int, default=1000)
    ap.add_argument("--rows", type=int, default=16)
    ap.add_argument("--out", help="gpu phase: where to write the recorded GPU states (.npz)")
    ap.add_argument("--gpu", help="cpu phase: the .npz the gpu phase wrote")
    args = ap.parse_args()
    if args.phase == "gpu" and not args.out:
        ap.error("the gpu phase needs --out")
    if args.phase == "cpu" and not args.gpu:
        ap.error("the cpu phase needs --gpu")
    run_gpu(args) if args.phase == "gpu" else run_cpu(args)


if __name__ == "__main__":
    main()
