"""Leapfrog (kick-drift-kick) integrator, mirror of
gfn/integrators/symplectic/leapfrog.py on the B200 kernels."""
import torch.nn as nn

from ._lib import GfnError, require_cuda
from .cuda import ops


class LeapfrogIntegrator(nn.Module):
    """forward(x, v, force, dt_scale, steps) -> (x, v) for one head.

    h = dt * dt_scale / 2; v_half = (v + h (F - Gamma(v))) / (1 + h mu(x));
    x += dt * dt_scale * v_half; v = (v_half + h (F - Gamma(v_half))) / (1 + h mu(x))
    with mu(x) = 5 sigmoid(x Wf^T + bf) from W_forget_stack / b_forget_stack
    (gfn/integrators/symplectic/leapfrog.py:24-118).
    """

    def __init__(self, christoffel, dt=0.01):
        super().__init__()
        self.christoffel = christoffel
        self.dt = dt

    def forward(self, x, v, force=None, dt_scale=1.0, steps=1, collect_christ=False, **kwargs):
        require_cuda(x, v, force)
        topology = kwargs.get("topology", 0)
        if topology != 0:
            raise GfnError("toroidal leapfrog is not implemented on this build")
        Wf = kwargs.get("W_forget_stack", None)
        bf = kwargs.get("b_forget_stack", None)
        if Wf is not None and Wf.dim() == 3:
            Wf = Wf[0]
        if bf is not None and bf.dim() == 2:
            bf = bf[0]
        if Wf is None or bf is None:
            # Without explicit stacks the reference takes mu from the
            # Christoffel's own gates: 5 sigmoid(forget_gate(x) + input_gate(F))
            # (gfn/geometry/lowrank.py:114-123).  With F == 0 that is the
            # forget gate alone; the input-gate term is not implemented.
            gate = getattr(self.christoffel, "forget_gate", None)
            if gate is None:
                Wf = bf = None
            elif force is None or not force.any():
                Wf, bf = gate.weight, gate.bias
            else:
                raise GfnError("leapfrog with the input-gate friction term (no W_forget_stack "
                               "given, non-zero force) is not implemented on this build")
        U = getattr(self.christoffel, "U", None)
        W = getattr(self.christoffel, "W", None)
        if U is None or W is None:
            raise GfnError("LeapfrogIntegrator needs a low-rank Christoffel (U, W)")
        return ops.leapfrog_fused(x, v, force, U, W, self.dt, dt_scale, steps, topology=0,
                                  Wf=Wf, bf=bf)
