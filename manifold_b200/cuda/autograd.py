"""Autograd functions of the single-head operators (the reference's
gfn/cuda/autograd.py: ChristoffelFusedFn, LeapfrogFusedFn).  Forward and
backward both run the library's kernels; the backward of the leapfrog is a
reverse replay that returns the gradients of every operand, the friction
gate's weights included."""
import torch
from torch.autograd import Function

from . import ops


class ChristoffelFusedFn(Function):
    """gfn/cuda/autograd.py:17-36."""

    @staticmethod
    def forward(ctx, v, U, W, x, V_w, plasticity, sing_thresh, sing_strength, topology, R, r):
        ctx.save_for_backward(v, U, W, x)
        ctx.args = (plasticity, sing_thresh, sing_strength, topology, R, r)
        return ops._christoffel_forward(v, U, W, x, V_w, plasticity, sing_thresh, sing_strength,
                                        topology, R, r)

    @staticmethod
    def backward(ctx, grad_gamma):
        v, U, W, x = ctx.saved_tensors
        gv, gU, gW, gx, _ = ops.christoffel_backward(grad_gamma.contiguous(), v, U, W, x, None, *ctx.args)
        return gv, gU, gW, gx, None, None, None, None, None, None, None


def christoffel_fused_autograd(v, U, W, x=None, V_w=None, plasticity=0.0, sing_thresh=1.0,
                               sing_strength=1.0, topology=0, R=2.0, r=1.0):
    return ChristoffelFusedFn.apply(v, U, W, x, V_w, plasticity, sing_thresh, sing_strength, topology,
                                    R, r)


class LeapfrogFusedFn(Function):
    """gfn/cuda/autograd.py:74-101, with the friction gate (Wf, bf), the input
    gate (Wi) and a tensor dt_scale differentiated too."""

    @staticmethod
    def forward(ctx, x, v, f, U, W, dt, dt_scale, steps, topology, Wf, bf, plasticity, R, r, Wi):
        ctx.save_for_backward(x, v, f, U, W, Wf, bf, Wi)
        ctx.args = (dt, dt_scale, steps, topology, R, r)
        return ops._leapfrog_forward(x, v, f, U, W, dt, dt_scale, steps, topology, Wf, bf, plasticity,
                                     R, r, Wi)

    @staticmethod
    def backward(ctx, grad_xn, grad_vn):
        x, v, f, U, W, Wf, bf, Wi = ctx.saved_tensors
        dt, dt_scale, steps, topology, R, r = ctx.args
        want_dt = isinstance(dt_scale, torch.Tensor) and ctx.needs_input_grad[6]
        dts = dt_scale.detach() if isinstance(dt_scale, torch.Tensor) else dt_scale
        out = ops.leapfrog_backward(grad_xn, grad_vn, x, v, f, U, W, dt, dts, steps, topology, R,
                                    r, Wf=Wf, bf=bf, Wi=Wi, want_dt=want_dt)
        gdt = None
        if want_dt:
            gdt = out.pop().reshape(dt_scale.shape).to(dt_scale.dtype)
        gx, gv, gf, gU, gW = out[:5]
        rest = out[5:]
        gWf = gbf = gWi = None
        if Wf is not None:
            gWf, gbf = rest[0], rest[1]
            rest = rest[2:]
            if bf is None:
                gbf = None
        if Wi is not None:
            gWi = rest[0]
        return (gx, gv, gf, gU, gW, None, gdt, None, None, gWf, gbf, None, None, None, gWi)


def leapfrog_fused_autograd(x, v, f, U, W, dt, dt_scale, steps, topology=0, Wf=None, bf=None,
                            plasticity=0.0, R=2.0, r=1.0, Wi=None):
    return LeapfrogFusedFn.apply(x, v, f, U, W, dt, dt_scale, steps, topology, Wf, bf, plasticity, R,
                                 r, Wi)
