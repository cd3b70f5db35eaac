"""Recurrent tokens/sec of the leapfrog recurrence on B200.

Default workload (N=1): the batched-decode configuration C4 -- 4,096
independent streams, d=1024, 24 layers, 16 heads, rank 64 (per-head 4),
leapfrog dt=0.1, uniform token ids over 32,000, persistent (x, v) state; one
step = one decode token for every stream through all 24 layers.  Weights are
seeded random (U, W ~ N(0, 0.2^2) etc.); data is synthetic.

Multi-GPU (torchrun): C4 shards its 4,096 streams over the ranks (strong
scaling: 4096 / N per GPU); the other configs give every rank its own batch
(weak scaling).  Rows are independent: no collective on the path, except the
gradient all-reduce of the training config C5.  Time is the max over ranks
of the device time.

--impl reference times the CPU baseline: the numpy restatement of the
reference's algorithm (oracle/), all host threads, on the same config.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: model shape, per-rank batch, default chunk (tokens per step)
    "c2": dict(V=2, d=256, NL=6, H=8, rank=32, B=64, dt=0.1, chunk=2000, parity=True,
               workload="C2 long-horizon recurrence fp32: d=256, 6 layers, 8 heads, rank 32, "
                        "leapfrog, batch 64, 100k-token stream in chunks"),
    "c4": dict(V=32000, d=1024, NL=24, H=16, rank=64, B=4096, dt=0.1, chunk=1, parity=False,
               strong=True,
               workload="C4 batched decode fp32: 4096 streams sharded over the GPUs, d=1024, "
                        "24 layers, 16 heads, rank 64, one token per step"),
    "c3_scan": dict(V=50257, d=512, NL=12, H=8, rank=32, B=256, dt=0.1, chunk=2048, functional=True,
                    scan=True,
                    workload="C3 LM prefill through the parallel-scan path (use_scan=True: "
                             "ParallelMLayer x 12, d=512, 8 heads), functional-embedding forces, "
                             "batch 256, L=2048"),
    "c3": dict(V=50257, d=512, NL=12, H=8, rank=32, B=256, dt=0.1, chunk=64, functional=True,
               workload="C3 LM prefill: bf16 functional-embedding forces, fp32 state, d=512, "
                        "12 layers, 8 heads, batch 256"),
    "c5": dict(V=32000, d=512, NL=8, H=8, rank=32, B=64, dt=0.1, chunk=1024, train=True,
               workload="C5 BPTT training step fp32: d=512, 8 layers, 8 heads, rank 32, leapfrog, "
                        "batch 64 per GPU, L=1024, Zipf ids over 32000, next-token CE, Adam; "
                        "NCCL gradient all-reduce when N > 1"),
    "c1": dict(V=2, d=128, NL=4, H=4, rank=16, B=32, dt=0.1, chunk=20, parity=True,
               workload="C1 cumulative parity fp32: d=128, 4 layers, 4 heads, batch 32, L=20"),
}


def flops_per_token(c):
    d, H = c["d"], c["H"]
    hd = d // H
    r = max(4, c["rank"] // H)
    # mixing 2 GEMVs (2*d*d MAC) + 2 friction GEMVs per head (2*hd*hd MAC per head)
    # + 2 Gamma evaluations (2 * 2*hd*r MAC per head) + ~30 elementwise flops per element
    mac = 2 * d * d + H * (2 * hd * hd + 4 * hd * r)
    return c["NL"] * (2 * mac + 30 * d)


def rank_batch(c, world):
    """Rows per rank: C4's streams are a fixed total sharded over the ranks
    (strong scaling); every other config gives each rank its own batch."""
    if c.get("batch_override"):
        return c["batch_override"]
    if c.get("strong"):
        if c["B"] % world:
            raise SystemExit(f"{c['B']} streams do not shard evenly over {world} GPUs")
        return c["B"] // world
    return c["B"]


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), hw=parts[5], hwt=parts[6],
                                 swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for k, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                            ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[k].lower().startswith("active"):
                    reasons.add(name)
        return dict(sm_mhz=float(np.median([r["sm"] for r in rows])), sm_max_mhz=rows[0]["max"],
                    samples=len(rows), reasons=sorted(reasons))


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def make_model(c, device):
    import torch
    import manifold_b200 as gfn
    from tests.golden import cases as C
    cfg = dict(c, seed=1234)
    P = C.make_params(cfg)
    torch.manual_seed(0)
    m = gfn.Manifold(**C.model_kwargs(cfg)).to(device).eval()
    C.load_into_model(m, cfg, P)
    for p in m.parameters():
        p.requires_grad_(False)
    return m, P


def make_ids(c, B, T, seed):
    from tests.golden import cases as C
    rng = np.random.default_rng(seed)
    if c.get("parity"):
        return rng.integers(0, 2, (B, T)).astype(np.int64)
    if c.get("functional"):
        return C.zipf_ids(rng, c["V"], (B, T))
    return rng.integers(0, c["V"], (B, T)).astype(np.int64)


def run_train(args, c):
    """One step = forward (trajectory stored) + readout + next-token CE +
    BPTT backward + gradient all-reduce (N > 1) + Adam step."""
    import torch
    import torch.distributed as dist
    from manifold_b200.distributed import allreduce_gradients
    from tests.golden import cases as C
    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import manifold_b200 as gfn
    cfg = dict(c, seed=1234)
    P = C.make_params(dict(cfg, V=2))  # seeded layer weights; the embedding keeps its init
    torch.manual_seed(0)
    m = gfn.Manifold(**C.model_kwargs(cfg)).to(dev).train()
    for layer, lp in zip(m.layers, P["layers"]):
        C.load_into_layer(layer, cfg, lp)
    params = list(m.parameters())
    opt = torch.optim.Adam(params, lr=1e-4)
    B, T, V = c["B"], args.chunk or c["chunk"], c["V"]
    steps, warm = args.steps, args.warmup
    host = [torch.from_numpy(make_ids(c, B, T + 1, 100 * rank + i)).pin_memory() for i in range(steps + warm)]
    # the library's loss kernels (one read of the logits forward, one read and
    # one write backward) for the reference loop's nn.CrossEntropyLoss()
    ce = gfn.CrossEntropyLoss()
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)

    def step(i):
        ids = host[i].to(dev, non_blocking=True)
        logits = m(ids[:, :T])[0]
        loss = ce(logits.reshape(-1, V), ids[:, 1:].reshape(-1))
        loss.backward()
        if world > 1:
            allreduce_gradients(params)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for i in range(warm):
        step(i)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    # all ranks start the timed region together (after rank 0's sampler is up)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    losses = []
    for i in range(steps):
        flush.zero_()
        ev[i][0].record(stream)
        loss = step(warm + i)
        lv = loss.item()  # device -> host read of the step's result
        ev[i][1].record(stream)
        losses.append(lv)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop() if sampler else None
    ms = sum(a.elapsed_time(b) for a, b in ev)
    # per-kernel device time of the two recurrence kernels (a second timed
    # pass with CUDA events around each launch), for the latency roofline
    from manifold_b200 import training as TR
    TR.KERNEL_EVENTS = []
    for i in range(min(2, steps)):
        flush.zero_()
        step(warm + i)
    torch.cuda.synchronize(dev)
    kev, TR.KERNEL_EVENTS = TR.KERNEL_EVENTS, None
    kt = {"fwd": [], "bwd": []}
    for tag, a0, a1 in kev:
        kt[tag].append(a0.elapsed_time(a1))
    fwd_ms = float(np.mean(kt["fwd"])) if kt["fwd"] else None
    bwd_ms = float(np.mean(kt["bwd"])) if kt["bwd"] else None
    if os.environ.get("GFN_BENCH_DEBUG"):
        print(f"rank {rank} step ms {[round(a.elapsed_time(b), 1) for a, b in ev]}", file=sys.stderr)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    result = None
    if rank == 0:
        hbm, _, kind = measured_peaks()
        tokens = world * B * T * steps
        value = tokens / (ms / 1e3)
        result = {
            "metric": "recurrent tokens/sec (prefill+decode)",
            "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms / steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Zipf ids; seeded random weights)",
            "config": {"workload": c["workload"], "batch_per_gpu": B, "tokens_per_step": T,
                       "dim": c["d"], "layers": c["NL"], "heads": c["H"], "rank": c["rank"],
                       "l2": "flushed (256 MB write) between timed steps",
                       "parallelism": f"dp{world}"},
            "e2e": {"value": round(value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(B * (T + 1) * 8), "d2h_bytes_per_step": 4,
                    "note": "each timed step already copies its ids from pinned host memory and reads the loss back"},
            "gpu_launches": steps * 4,
            "roofline": c5_roofline(c, B, T, ms / steps, fwd_ms, bwd_ms, dev),
            "loss": [round(x, 4) for x in losses],
            "clocks": clocks,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def c5_roofline(c, B, T, step_ms, fwd_ms, bwd_ms, dev):
    """Training step roofline: the two recurrence kernels (84% of the step,
    profiles/launches_c5.md) are dependent chains over T tokens x NL layers.
    Floor of one layer step = the latency probe's dependent chain on this
    plan; the backward replays the forward chain and runs the reverse chain,
    so its floor is taken as twice that (a lower bound)."""
    from manifold_b200.cuda import ops
    r = max(4, c["rank"] // c["H"])
    plan = ops.leapfrog_plan(B, c["d"], c["H"], r, c["NL"])
    n = T * c["NL"]
    fwd_ns = fwd_ms * 1e6 / n if fwd_ms else None
    lat = latency_floor(dev, r, plan["clusters"], fwd_ns or 1.0)
    floor = lat["floor_ns_per_layer_step"]
    bwd_ns = bwd_ms * 1e6 / n if bwd_ms else None
    out = {"bound": "latency", "kernel": "leapfrog_bwd_kernel", "unit": "ns per layer step",
           "achieved": round(bwd_ns, 1) if bwd_ns else None, "peak": round(2 * floor, 1),
           "frac": round(2 * floor / bwd_ns, 4) if bwd_ns else None, "traffic": None,
           "forward": {"kernel": "leapfrog_seq_kernel (training)", "ms_per_launch": fwd_ms,
                       "ns_per_layer_step": round(fwd_ns, 1) if fwd_ns else None,
                       "floor_ns": floor, "frac": round(floor / fwd_ns, 4) if fwd_ns else None},
           "backward": {"ms_per_launch": bwd_ms, "floor_ns": round(2 * floor, 1),
                        "floor_note": "forward replay + reverse chain, each at least the probe floor"},
           "share_of_step": round(((fwd_ms or 0) + (bwd_ms or 0)) / step_ms, 3),
           "latency_probe": lat["source"]}
    return out


def run_ours(args, c):
    import torch
    import torch.distributed as dist
    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from manifold_b200.cuda import ops
    m, P = make_model(c, dev)
    B, T = rank_batch(c, world), args.chunk or c["chunk"]
    steps, warm = args.steps, args.warmup
    ids_host = [torch.from_numpy(make_ids(c, B, T, 100 * rank + i)).pin_memory()
                for i in range(steps + warm)]
    ids_dev = [t.to(dev) for t in ids_host]
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    if args.path != "auto":
        m.recurrence_path = args.path
    if args.mixing != "default":
        ops.set_layered_mixing({"split_bf16": ops.MIX_SPLIT_BF16, "split_f16": ops.MIX_SPLIT_F16,
                                "fp32": ops.MIX_FP32_SIMT, "umma_f16": ops.MIX_UMMA_F16}[args.mixing])
    layered = m._use_layered(B)
    packed, meta = m._pack.get(list(m.layers), layered=layered)
    seqfn = ops.leapfrog_layered_sequence if layered else ops.leapfrog_sequence
    if c.get("functional"):
        m.force_dtype = torch.bfloat16

    x = m.x0.detach().expand(B, -1).contiguous()
    v = m.v0.detach().expand(B, -1).contiguous()
    want_v = True

    def step(i, state):
        with torch.no_grad():
            if c.get("functional"):
                forces = m.embedding(ids_dev[i], out_dtype=torch.bfloat16)
                xs, vs, xf, vf = seqfn(state[0], state[1], packed, meta, c["dt"],
                                       forces=forces, want_v_seq=want_v)
            else:
                xs, vs, xf, vf = seqfn(state[0], state[1], packed, meta, c["dt"],
                                       ids=ids_dev[i], table=m.embedding.weight,
                                       want_v_seq=want_v)
        return (xf, vf)

    state = (x, v)
    for i in range(warm):
        state = step(i, state)
    torch.cuda.synchronize(dev)
    if args.phase_profile:
        return phase_profile(step, warm, state, dev)
    # kernel-level event timing of the sequence kernel: per step, L2 flushed between
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    # all ranks start the timed region together (after rank 0's sampler is up)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    wall0 = time.perf_counter()
    for i in range(steps):
        flush.zero_()
        ev[i][0].record(stream)
        state = step(warm + i, state)
        ev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - wall0
    ms = sum(a.elapsed_time(b) for a, b in ev)
    # end to end through the public API: pinned host ids -> device, recurrence,
    # final state read back to the host, every step
    # the step's output x (the state the readout consumes; v is carried state
    # that stays on the device) is read back on a copy stream into alternating
    # pinned buffers, so step i's readback overlaps step i+1's kernels (every
    # step's output still reaches the host; the timed region ends after the
    # last copy)
    hbufs = [torch.empty(B, c["d"], dtype=torch.float32).pin_memory() for _ in range(2)]
    copy_stream = torch.cuda.Stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = (x, v)

    def e2e_step(i, st):
        with torch.no_grad():
            idd = ids_host[i].to(dev, non_blocking=True)
            _, _, st, _ = m.recurrence(idd, state=st)
        done = torch.cuda.Event()
        done.record(stream)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(done)
            hbufs[i % 2].copy_(st[0], non_blocking=True)
            st[0].record_stream(copy_stream)
        return st

    for i in range(warm):  # the public-API path has its own first-call costs
        st = e2e_step(i, st)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for i in range(steps):
        st = e2e_step(warm + i, st)
    stream.wait_stream(copy_stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    clocks = sampler.stop() if sampler else None
    # per-kernel CUDA-event timing of the layered path (a second timed pass with
    # events recorded around every head-step and mixing launch on their stream)
    ktime = layered_kernel_times(step, warm, state, steps, flush, dev) if layered else None
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    tokens = world * B * T * steps
    value = tokens / (ms / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)
    result = None
    if rank == 0:
        hbm, bf16, peak_kind = measured_peaks()
        step_ms = ms / steps
        # algorithmic HBM bytes per launch: ids (8 B) + x_seq, v_seq writes (8 d B) per
        # token-row, the packed weights once, the state in/out
        per_tok = (2 if c.get("functional") else 8) * (c["d"] if c.get("functional") else 1) \
            + 4 * c["d"] * (2 if want_v else 1)
        alg = B * T * per_tok + packed.numel() * 4 + 4 * 4 * B * c["d"]
        achieved = alg / (step_ms / 1e3) / 1e9
        fl = flops_per_token(c) * B * T / (step_ms / 1e3) / 1e12
        plan = ops.leapfrog_plan(B, c["d"], c["H"], max(4, c["rank"] // c["H"]), c["NL"])
        layer_step_ns = step_ms * 1e6 / (T * c["NL"])
        latency = None if layered else latency_floor(dev, max(4, c["rank"] // c["H"]),
                                                     plan["clusters"], layer_step_ns)
        result = {
            "metric": "recurrent tokens/sec (prefill+decode)",
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warm,
            "ms_per_step": round(ms / steps, 4),
            "higher_is_better": True,
            "scaling": "strong" if c.get("strong") else "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded parity bits / ids; seeded random weights)",
            "config": {"workload": c["workload"], "batch_per_gpu": B, "tokens_per_step": T,
                       "dim": c["d"], "layers": c["NL"], "heads": c["H"],
                       "rank": c["rank"], "l2": "flushed (256 MB write) between timed steps",
                       "plan": plan},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(B * T * 8), "d2h_bytes_per_step": int(B * c["d"] * 4),
                    "read_back": "the step's output x [B, d] (v stays on the device as carried state)"},
            "gpu_launches": steps * ((2 * c["NL"] + 2) * T if layered else 1)
            + (steps if c.get("functional") else 0),
            "recurrence_path": "layered (head-step kernel + split-precision tensor-core mixing GEMM per layer)"
            if layered else "fused persistent cluster kernel",
            "roofline": roofline_entry(c, layered, achieved, hbm, bf16, peak_kind, fl, step_ms, T,
                                       latency, ktime, B),
            "clocks": clocks,
            "wall_s_timed": round(wall, 3),
        }
        if not args.no_cpu_baseline and world == 1:
            result["cpu_baseline"] = cpu_baseline(c, args.cpu_tokens)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_scan(args, c):
    """C3 through the parallel-scan path (use_scan=True): one step = the 12
    ParallelMLayers over one [B, L] batch of functional-embedding forces
    (LayerNorm + the three d x d projections as one split-fp16 tcgen05 GEMM +
    the fused sigmoid/softplus/two-scan kernel per layer)."""
    import torch
    import torch.distributed as dist
    import manifold_b200 as gfn
    from manifold_b200.cuda import ops
    from tests.golden import cases as C
    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    kw = dict(C.model_kwargs(dict(c, seed=1234)), use_scan=True)
    m = gfn.Manifold(**kw).to(dev).eval()
    B, T, d = c["B"], args.chunk or c["chunk"], c["d"]
    steps, warm = args.steps, args.warmup
    ids_host = [torch.from_numpy(make_ids(c, B, T, 100 * rank + i)).pin_memory() for i in range(steps + warm)]
    ids_dev = [t.to(dev) for t in ids_host]
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)

    def layers(forces):
        cur = forces
        for layer in m.layers:
            cur, _, _, _ = layer(None, None, force=cur)
        return cur

    def step(i):
        with torch.no_grad():
            return layers(m.embedding(ids_dev[i]))

    for i in range(warm):
        step(i)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        ev[i][0].record(stream)
        step(warm + i)
        ev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    ms = sum(a.elapsed_time(b) for a, b in ev)
    # end to end: ids from pinned host memory, the layers, the last position's
    # state read back to the host
    hx = torch.empty(B, d, dtype=torch.float32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        with torch.no_grad():
            out = layers(m.embedding(ids_host[warm + i].to(dev, non_blocking=True)))
        hx.copy_(out[:, -1], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    # the fused layer-scan kernel alone, per launch (CUDA events on its stream)
    layer = m.layers[0]
    with torch.no_grad():
        f = layer.norm_x(m.embedding(ids_dev[0]))
        Wcat = torch.cat([layer.to_A[0].weight, layer.to_dt[0].weight, layer.to_B.weight], 0)
        bcat = torch.cat([layer.to_A[0].bias, layer.to_dt[0].bias, layer.to_B.bias], 0)
        z = torch.nn.functional.linear(f, Wcat, bcat)
        ks = []
        for i in range(max(3, steps)):
            flush.zero_()
            k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            k0.record(stream)
            ops.parallel_layer_scan(z, layer.heads, layer.base_dt)
            k1.record(stream)
            ks.append((k0, k1))
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        from manifold_b200.readout import SplitLinear
        fl = f.reshape(-1, d)
        for i in range(steps):
            SplitLinear.apply(layer.norm_x(fl), Wcat, bcat)
        g1.record(stream)
    torch.cuda.synchronize(dev)
    scan_us = sum(a.elapsed_time(b) for a, b in ks) * 1e3 / len(ks)
    proj_us = g0.elapsed_time(g1) * 1e3 / steps
    clocks = sampler.stop() if sampler else None
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    result = None
    if rank == 0:
        hbm, bf16, peak_kind = measured_peaks()
        tokens = world * B * T * steps
        scan_bytes = 20.0 * B * T * d  # read z [B, L, 3d], write x_seq, v_seq
        scan_gbs = scan_bytes / (scan_us * 1e-6) / 1e9
        proj_tf = 2.0 * B * T * d * 3 * d / (proj_us * 1e-6) / 1e12
        result = {
            "metric": "recurrent tokens/sec (prefill+decode)", "value": round(tokens / (ms / 1e3), 1),
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": round(ms / steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Zipf ids; seeded random weights)",
            "config": {"workload": c["workload"], "batch_per_gpu": B, "tokens_per_step": T, "dim": d,
                       "layers": c["NL"], "heads": c["H"], "l2": "flushed (256 MB write) between timed steps"},
            "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(B * T * 8), "d2h_bytes_per_step": int(B * d * 4)},
            "gpu_launches": steps * (1 + c["NL"]),
            "recurrence_path": "parallel scan (ParallelMLayer: LayerNorm + projection GEMM + fused scan kernel)",
            "roofline": {"bound": "hbm", "kernel": "parallel_layer_scan_kernel", "achieved": round(scan_gbs, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(scan_gbs / hbm, 4),
                         "traffic": TRAFFIC.get((c.get("name"), "scan")), "peak_source": peak_kind,
                         "launch_us": round(scan_us, 2),
                         "algorithmic_bytes_per_launch": scan_bytes,
                         "projections": {"launch_us": round(proj_us, 2), "tflops": round(proj_tf, 1),
                                         "note": "LayerNorm + [B*L, d] x [d, 3d] product as the split-fp16 "
                                                 "tcgen05 GEMM (tflops: the fp32 product's FLOPs; the tensor "
                                                 "pipe runs 3x, plus the operand split)"}},
            "clocks": clocks,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def latency_floor(dev, rank, clusters, layer_step_ns, steps=20000):
    """Latency roof of the fused recurrence: ns per layer step of the
    dependent chain alone (gfn_debug_latency_probe: the reductions, kick
    arithmetic and the two cluster exchanges of a layer step, no weight
    traffic), on the plan's cluster count, against the measured layer step."""
    import ctypes
    import torch
    from manifold_b200 import _lib
    buf = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    _lib.call("gfn_debug_latency_probe", rank, clusters, 100, ctypes.c_void_p(buf.data_ptr()),
              stream.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    _lib.call("gfn_debug_latency_probe", rank, clusters, steps, ctypes.c_void_p(buf.data_ptr()),
              stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    floor_ns = e0.elapsed_time(e1) * 1e6 / steps
    return {"floor_ns_per_layer_step": round(floor_ns, 1),
            "achieved_ns_per_layer_step": round(layer_step_ns, 1),
            "frac": round(floor_ns / layer_step_ns, 4),
            "floor_cycles_per_layer_step": round(buf.item() / steps, 1),
            "source": "gfn_debug_latency_probe (dependent chain of one layer step, no weight traffic)"}


def layered_kernel_times(step, i0, state, steps, flush, dev):
    """Average device time per launch of the layered path's head-step and
    mixing kernels: CUDA events recorded by the library around each launch,
    on the launching stream, over `steps` steps (L2 flushed between steps)."""
    import ctypes
    import torch
    from manifold_b200 import _lib
    _lib.call("gfn_debug_layered_timing", 1)
    try:
        for i in range(steps):
            flush.zero_()
            state = step(i0 + i, state)
        torch.cuda.synchronize(dev)
        hm, mm, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
        _lib.call("gfn_debug_layered_timing_read", ctypes.addressof(hm), ctypes.addressof(mm),
                  ctypes.addressof(n))
    finally:
        _lib.call("gfn_debug_layered_timing", 0)
    n = max(1, n.value)
    return dict(head_us=hm.value * 1e3 / n, mix_us=mm.value * 1e3 / n, launches=n)


# DRAM bytes (read + write) per launch of the dominant kernels, from one ncu
# capture each (dram__bytes_read.sum + dram__bytes_write.sum; the commands and
# figures are in profiles/*.md).  Keyed by (config, kernel).
TRAFFIC = {
    ("c4", "head"): 49.88e6 + 8.12e6,  # profiles/head_umma_c4.md
    ("c4", "mix"): 42.57e6 + 0.64e6,   # profiles/mix_umma_c4.md
}


def roofline_entry(c, layered, achieved_gbs, hbm, bf16, peak_kind, fp32_tflops, step_ms, T, latency,
                   ktime=None, B=None):
    """Roofline of the recurrence.

    Layered path: the dominant kernel of the step, timed per launch with CUDA
    events.  Mixing GEMM: algorithmic FLOPs = the fp32 product 2 * 2 * B * d^2
    per launch (x and v; the split-fp16 scheme issues three times this on the
    tensor pipe) against the measured bf16 peak.  Head step: algorithmic
    bytes = read x, v, force + write x', v' (20 B per element of [B, d]) against
    the measured copy bandwidth.  Fused path: algorithmic HBM bytes of the
    launch against the copy bandwidth (tiny by construction: the chain is
    latency-bound) plus the latency roof from the probe kernel."""
    if layered and ktime:
        d = c["d"]
        mix_fl = 2.0 * 2 * B * d * d
        head_bytes = 20.0 * B * d
        mix_tf = mix_fl / (ktime["mix_us"] * 1e-6) / 1e12
        head_gbs = head_bytes / (ktime["head_us"] * 1e-6) / 1e9
        step_tf = flops_per_token(c) * B * T / (step_ms / 1e3) / 1e12
        kernels = {
            "mixing_gemm": {"kernel": "mix_umma_kernel (tcgen05, split-fp16)", "launch_us": round(ktime["mix_us"], 2),
                            "algorithmic_flop_per_launch": mix_fl, "achieved_tflops": round(mix_tf, 1),
                            "frac_of_bf16_peak": round(mix_tf / bf16, 4),
                            "tensor_pipe_tflops": round(3 * mix_tf, 1),
                            "traffic": TRAFFIC.get((c.get("name"), "mix"))},
            "head_step": {"kernel": "layered_head_umma_kernel (tcgen05 gate, 64-row tiles)",
                          "launch_us": round(ktime["head_us"], 2),
                          "algorithmic_bytes_per_launch": head_bytes, "achieved_gbs": round(head_gbs, 1),
                          "frac_of_hbm": round(head_gbs / hbm, 4),
                          "traffic": TRAFFIC.get((c.get("name"), "head"))},
        }
        if ktime["mix_us"] >= ktime["head_us"]:
            k = kernels["mixing_gemm"]
            top = {"bound": "tensor", "kernel": "mixing_gemm", "achieved": k["achieved_tflops"], "peak": bf16,
                   "unit": "TFLOP/s", "frac": k["frac_of_bf16_peak"], "traffic": k["traffic"]}
        else:
            k = kernels["head_step"]
            top = {"bound": "hbm", "kernel": "head_step", "achieved": k["achieved_gbs"], "peak": hbm,
                   "unit": "GB/s", "frac": k["frac_of_hbm"], "traffic": k["traffic"]}
        top.update({"peak_source": peak_kind, "kernels": kernels, "layer_steps_timed": ktime["launches"],
                    "step": {"algorithmic_fp32_tflops": round(step_tf, 2),
                             "frac_of_bf16_peak": round(step_tf / bf16, 4),
                             "note": "all algorithmic fp32 FLOPs of the step (mixing, friction, Gamma, "
                                     "elementwise) over the whole step time"}})
        return top
    return {"bound": "hbm", "achieved": round(achieved_gbs, 2), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved_gbs / hbm, 5), "traffic": TRAFFIC.get((c.get("name"), "seq")),
            "peak_source": peak_kind,
            "note": "dependent chain: HBM is not the binding roof; see latency",
            "fp32_tflops": round(fp32_tflops, 3), "latency": latency}


def phase_profile(step, i, state, dev):
    """Cycles per layer step spent in each phase by CTA 0 (clock64 counters)."""
    import ctypes
    import torch
    from manifold_b200 import _lib
    buf = torch.zeros(12, dtype=torch.int64, device=dev)
    _lib.call("gfn_debug_set_phase_profile", ctypes.c_void_p(buf.data_ptr()))
    step(i, state)
    torch.cuda.synchronize(dev)
    _lib.call("gfn_debug_set_phase_profile", None)
    v = buf.tolist()
    n = max(1, v[11])
    names = ["head_wait", "head_step_and_send", "exchange_wait", "mixing_compute",
             "reduce_and_sync", "norm_exchange", "norm", "token_io", "mixing_chunk_wait"]
    out = {nm: round(v[k] / n, 1) for k, nm in enumerate(names)}
    out["total"] = round(sum(v[:9]) / n, 1)
    return {"phase_cycles_per_layer_step": out, "layer_steps": n}


def cpu_baseline(c, tokens):
    """The numpy port of the reference algorithm (oracle/) on the host cores,
    on a bounded sample of the same workload."""
    from oracle import gfn_oracle as O
    from tests.golden import cases as C
    cfg = dict(c, seed=1234)
    P = C.make_params(cfg)
    B = c["B"]
    T = tokens or max(1, min(c.get("chunk", 1), 200))
    Bs = B if B <= 256 else 256
    ids = make_ids(c, Bs, T, 7)
    F = O.functional_embedding(ids, P["func"]) if c.get("functional") else P["emb"][ids]
    x0 = np.broadcast_to(P["x0"], (Bs, c["d"])).copy()
    v0 = np.broadcast_to(P["v0"], (Bs, c["d"])).copy()
    t0 = time.perf_counter()
    O.manifold_forward(x0, v0, F, P["layers"], c["H"], c["dt"])
    dt = time.perf_counter() - t0
    return {"value": round(Bs * T / dt, 1), "unit": "tokens/s", "cores": os.cpu_count(),
            "kind": "port", "sample": f"{Bs} rows x {T} tokens through all {c['NL']} layers "
                                      f"(numpy float32, BLAS threads = host cores)"}


def run_reference(args, c):
    world, rank, _ = dist_env()
    if rank != 0:
        return None
    T = args.cpu_tokens or max(1, min(c.get("chunk", 1), 100))
    vals = []
    for _ in range(args.warmup):
        cpu_baseline(c, T)
    for _ in range(args.steps):
        vals.append(cpu_baseline(c, T)["value"])
    v = float(np.mean(vals))
    B = c["B"] if c["B"] <= 256 else 256
    cb = {"value": round(v, 1), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
          "sample": f"{B} rows x {T} tokens per step, all {c['NL']} layers, numpy float32"}
    return {"metric": "recurrent tokens/sec (prefill+decode)", "value": round(v, 1),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(B * T / v * 1e3, 3), "higher_is_better": True,
            "scaling": "strong" if c.get("strong") else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": c["workload"], "batch_per_gpu": c["B"]},
            "cpu_baseline": cb,
            "e2e": {"value": round(v, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS))
    ap.add_argument("--chunk", type=int, default=0, help="tokens per step (default per config)")
    ap.add_argument("--batch", type=int, default=0,
                    help="rows per GPU (default: the config's; C4 shards its 4096 streams)")
    ap.add_argument("--cpu-tokens", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--path", default="auto", choices=["auto", "fused", "layered"],
                    help="recurrence path (auto: by batch size)")
    ap.add_argument("--mixing", default="default", choices=["default", "umma_f16", "split_bf16", "split_f16", "fp32"],
                    help="layered path's mixing GEMM arithmetic (default: the library's)")
    ap.add_argument("--phase-profile", action="store_true",
                    help="print per-phase cycle counts of CTA 0 for one step instead")
    args = ap.parse_args()
    c = dict(CONFIGS[args.config], name=args.config)
    if args.batch:
        c["batch_override"] = args.batch
    if args.impl == "reference":
        out = run_reference(args, c)
    else:
        out = run_train(args, c) if c.get("train") else run_scan(args, c) if c.get("scan") \
            else run_ours(args, c)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
