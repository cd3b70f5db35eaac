"""Training path: BPTT through the fused recurrence.

The reference gets these gradients from torch autograd over its per-token
loop (gfn/model.py:377-402 in train mode).  Here one forward launch stores
every layer step's input state, one reverse launch replays the steps and
emits per-step gradient factors, and the parameter gradients are formed from
those factors with batched GEMMs / sums (cuBLAS via torch, deterministic).
"""
import ctypes

import torch

from . import _lib
from ._lib import GfnError, call, ptr, require_cuda
from .packing import layer_tensors

NSIG = 11
NSMALL = 4


def _stacks(layers):
    U, W, Wf, bf, dtp, mix = layer_tensors(layers)
    out = [torch.stack(U), torch.stack(W), torch.stack(Wf), torch.stack(bf), torch.cat(dtp)]
    if mix:
        out += [torch.stack([m[i] for m in mix]) for i in range(6)]
    return out


# Measurement hook: when a list, each forward / backward recurrence launch
# appends ("fwd" | "bwd", start event, end event), CUDA events recorded on the
# launch stream around the kernel (bench.py's C5 roofline reads them).
KERNEL_EVENTS = None


def _mark(tag, stream):
    """An event on the current stream (the stream the library launches on)."""
    if KERNEL_EVENTS is None:
        return None
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    return e


class LeapfrogSequenceTrain(torch.autograd.Function):
    """(x0, v0, forces, *param stacks) -> (x_seq, v_seq, x_final, v_final)."""

    @staticmethod
    def forward(ctx, meta, mask, x0, v0, forces, *stacks):
        d, H, r, NL = meta["dim"], meta["heads"], meta["rank"], meta["num_layers"]
        base_dt = meta["base_dt"]
        B, L, _ = forces.shape
        dev = forces.device
        f32 = lambda t: None if t is None else t.detach().to(torch.float32).contiguous()
        st = [f32(t) for t in stacks]
        n = _lib.load().gfn_leapfrog_pack_train_floats(d, H, r, NL)
        if n < 0:
            raise GfnError("unsupported shapes for training")
        packed = torch.empty(int(n), device=dev, dtype=torch.float32)
        mix = st[5:] if len(st) > 5 else [None] * 6
        stream = _lib.stream_of(dev)
        call("gfn_leapfrog_pack_train", *[ptr(t) for t in st[:5]], *[ptr(t) for t in mix], d, H, r, NL,
             ptr(packed), packed.numel(), stream)
        broadcast = x0.dim() == 1 or x0.shape[0] == 1
        x0c, v0c = f32(x0).reshape(-1, d), f32(v0).reshape(-1, d)
        if broadcast:
            x0c = x0c.expand(B, d).contiguous()
            v0c = v0c.expand(B, d).contiguous()
        fc = forces.detach().contiguous()
        fl32 = fc if fc.dtype == torch.float32 else None
        fbf = fc if fc.dtype == torch.bfloat16 else None
        m = f32(mask)
        x_seq = torch.empty(B, L, d, device=dev)
        v_seq = torch.empty_like(x_seq)
        xf = torch.empty(B, d, device=dev)
        vf = torch.empty_like(xf)
        # layer-step inputs (x, v), the mixing outputs (z_x, z_v) and the RMSNorm
        # factors (r_x, r_v) of every layer step, for the backward
        S = NL * L * B * d
        traj = torch.empty(4 * S + 2 * NL * L * B, device=dev)
        e0 = _mark("fwd", stream)
        call("gfn_leapfrog_sequence_forward_train", ptr(x0c), ptr(v0c), d, ptr(fl32), ptr(fbf), None,
             None, 0, ptr(m), ptr(packed), packed.numel(), B, L, d, H, r, NL, float(base_dt),
             ptr(x_seq), ptr(v_seq), ptr(xf), ptr(vf), ptr(traj), stream)
        if e0 is not None:
            KERNEL_EVENTS.append(("fwd", e0, _mark("fwd", stream)))
        ctx.save_for_backward(packed, traj, fc, *[t for t in st])
        ctx.mask = m
        ctx.meta = meta
        ctx.broadcast = broadcast
        ctx.shapes = (B, L)
        return x_seq, v_seq, xf, vf

    @staticmethod
    def backward(ctx, gxs, gvs, gxf, gvf):
        packed, traj, fc = ctx.saved_tensors[:3]
        st = ctx.saved_tensors[3:]
        meta = ctx.meta
        d, H, r, NL = meta["dim"], meta["heads"], meta["rank"], meta["num_layers"]
        base_dt = meta["base_dt"]
        B, L = ctx.shapes
        dev = fc.device
        c = lambda t: None if t is None else t.to(torch.float32).contiguous()
        gxs, gvs, gxf, gvf = c(gxs), c(gvs), c(gxf), c(gvf)
        n = _lib.load().gfn_leapfrog_backward_workspace_floats(B, L, d, H, r, NL)
        ws = torch.empty(int(n), device=dev)
        dx0 = torch.empty(B, d, device=dev)
        dv0 = torch.empty_like(dx0)
        dF = torch.empty(B, L, d, device=dev)
        fl32 = fc if fc.dtype == torch.float32 else None
        fbf = fc if fc.dtype == torch.bfloat16 else None
        bstream = _lib.stream_of(dev)
        e0 = _mark("bwd", bstream)
        call("gfn_leapfrog_sequence_backward", ptr(traj), ptr(fl32), ptr(fbf), None, None, 0,
             ptr(ctx.mask), ptr(packed), packed.numel(), ptr(gxs), ptr(gvs), ptr(gxf), ptr(gvf), B, L,
             d, H, r, NL, float(base_dt), ptr(dx0), ptr(dv0), ptr(dF), ptr(ws), ws.numel(), bstream)
        if e0 is not None:
            KERNEL_EVENTS.append(("bwd", e0, _mark("bwd", bstream)))
        grads = param_grads(ws, traj, st, B, L, d, H, r, NL, base_dt)
        if ctx.broadcast:
            dx0 = dx0.sum(0, keepdim=True)
            dv0 = dv0.sum(0, keepdim=True)
        return (None, None, dx0, dv0, dF.to(fc.dtype), *grads)


def param_grads(ws, traj, stacks, B, L, d, H, r, NL, base_dt):
    """Parameter gradients from the backward's per-step signals (see the
    workspace layout in include/gfn_b200.h)."""
    N = L * B
    S = NL * N * d
    hd = d // H
    sig = ws[: NSIG * S].view(NSIG, NL, N, d)
    x2, v2, dzx, dzv, sgx, sgv, dz1, dz2, vh, dg1, dg2 = sig.unbind(0)
    M = NL * N * H * r
    small = ws[NSIG * S: NSIG * S + NSMALL * M].view(NSMALL, NL, N, H, r)
    q1, q2, dp1, dp2 = small.unbind(0)
    deff = ws[NSIG * S + NSMALL * M: NSIG * S + NSMALL * M + NL * N * H].view(NL, N, H)
    xin = traj[:S].view(NL, N, d)
    vin = traj[S:2 * S].view(NL, N, d)
    hv = lambda t: t.view(NL, N, H, hd)
    dWf = torch.einsum("lnhj,lnhk->lhjk", hv(dz1), hv(xin)) + torch.einsum("lnhj,lnhk->lhjk", hv(dz2), hv(x2))
    dbf = (hv(dz1) + hv(dz2)).sum(1)
    dU = torch.einsum("lnhj,lnhr->lhjr", hv(vin), dp1) + torch.einsum("lnhj,lnhr->lhjr", hv(vh), dp2)
    dW = torch.einsum("lnhj,lnhr->lhjr", hv(dg1), q1) + torch.einsum("lnhj,lnhr->lhjr", hv(dg2), q2)
    theta = stacks[4].view(NL, H)
    ddt = deff.sum(1) * base_dt * torch.sigmoid(theta)
    out = [dU.reshape(NL * H, hd, r), dW.reshape(NL * H, hd, r), dWf.reshape(NL * H, hd, hd),
           dbf.reshape(NL * H, hd), ddt.reshape(NL * H)]
    if len(stacks) > 5:
        dWx = torch.bmm(dzx.transpose(1, 2), x2)
        dWv = torch.bmm(dzv.transpose(1, 2), v2)
        out += [dWx, dzx.sum(1), sgx.sum(1), dWv, dzv.sum(1), sgv.sum(1)]
    return out


def leapfrog_sequence_train(layers, x0, v0, forces, mask=None):
    """Differentiable fused recurrence over `layers` (MLayer list)."""
    require_cuda(x0, v0, forces, mask)
    l0 = layers[0]
    hd = l0.head_dim
    meta = dict(dim=l0.dim, heads=l0.heads, rank=l0.christoffels[0].U.shape[1],
                num_layers=len(layers), base_dt=l0.base_dt)
    if hd > 64:
        raise GfnError("training supports head_dim <= 64")
    return LeapfrogSequenceTrain.apply(meta, mask, x0, v0, forces, *_stacks(layers))


def manifold_train_forward(model, input_ids, attention_mask, state, force_manual):
    """Manifold.forward with autograd (gfn/model.py:142-402, train mode)."""
    forces = model._forces(input_ids, force_manual)
    if state is None:
        x, v = model.x0, model.v0
    else:
        x, v = state
    mask = None if attention_mask is None else attention_mask.to(torch.float32)
    x_seq, v_seq, xf, vf = leapfrog_sequence_train(list(model.layers), x, v, forces, mask)
    out = x_seq if model.holographic else model.readout_norm(x_seq)
    logits = model._apply_readout(out)
    return logits, (xf, vf), [], list(v_seq.unbind(1)), list(x_seq.unbind(1)), forces
