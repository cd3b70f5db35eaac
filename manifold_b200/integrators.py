"""Leapfrog (kick-drift-kick) integrator, mirror of
gfn/integrators/symplectic/leapfrog.py on the B200 kernels."""
import torch.nn as nn

from ._lib import GfnError, require_cuda
from .cuda import ops


class LeapfrogIntegrator(nn.Module):
    """forward(x, v, force, dt_scale, steps) -> (x, v) for one head.

    h = dt * dt_scale / 2; v_half = (v + h (F - Gamma(v))) / (1 + h mu(x));
    x += dt * dt_scale * v_half; v = (v_half + h (F - Gamma(v_half))) / (1 + h mu(x))
    with mu(x) = 5 sigmoid(x Wf^T + bf) from W_forget_stack / b_forget_stack,
    else from the Christoffel's own gates, 5 sigmoid(forget_gate(x) +
    input_gate(F)); on the torus (ToroidalChristoffel) Gamma is the toroidal
    term, the gate reads [sin x, cos x] and x wraps into [0, 2 pi)
    (gfn/integrators/symplectic/leapfrog.py:24-118).  Differentiable: the
    backward is the library's reverse replay.
    """

    def __init__(self, christoffel, dt=0.01):
        super().__init__()
        self.christoffel = christoffel
        self.dt = dt

    def forward(self, x, v, force=None, dt_scale=1.0, steps=1, collect_christ=False, **kwargs):
        require_cuda(x, v, force)
        topology = kwargs.get("topology", getattr(self.christoffel, "topology_id", 0))
        if topology == 0 and getattr(self.christoffel, "is_torus", False):
            topology = 1
        Wf = kwargs.get("W_forget_stack", None)
        bf = kwargs.get("b_forget_stack", None)
        Wi = None
        if Wf is not None and Wf.dim() == 3:
            Wf = Wf[0]
        if bf is not None and bf.dim() == 2:
            bf = bf[0]
        if Wf is None or bf is None:
            # Without explicit stacks the friction is the Christoffel's own
            # gate: 5 sigmoid(forget_gate(x) + input_gate(F))
            # (gfn/geometry/lowrank.py:114-123, gfn/geometry/toroidal.py:113-124).
            gate = getattr(self.christoffel, "forget_gate", None)
            if gate is None:
                Wf = bf = None
            else:
                Wf, bf = gate.weight, gate.bias
                ig = getattr(self.christoffel, "input_gate", None)
                if ig is not None and force is not None:
                    Wi = ig.weight
        U = getattr(self.christoffel, "U", None)
        W = getattr(self.christoffel, "W", None)
        if topology == 0 and (U is None or W is None):
            raise GfnError("LeapfrogIntegrator needs a low-rank Christoffel (U, W) or the torus")
        if topology == 1:
            R = getattr(self.christoffel, "R", 2.0)
            r = getattr(self.christoffel, "r", 1.0)
            return ops.leapfrog_fused(x, v, force, None, None, self.dt, dt_scale, steps, topology=1,
                                      Wf=Wf, bf=bf, R=R, r=r, Wi=Wi)
        return ops.leapfrog_fused(x, v, force, U, W, self.dt, dt_scale, steps, topology=0,
                                  Wf=Wf, bf=bf, Wi=Wi)
