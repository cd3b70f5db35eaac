"""Low-rank Christoffel geometry (mirror of gfn/geometry/lowrank.py and
gfn/geometry/reactive.py) on the B200 kernels.

The modules keep the reference's parameters, names and initialisation so a
reference state_dict loads unchanged.  The Euclidean, plasticity-free form
used by the leapfrog path runs on the GPU kernels; the other branches of the
reference (torus features, plasticity, singularities) raise.
"""
import torch
import torch.nn as nn

from ._lib import GfnError, require_cuda
from .cuda import ops


class LowRankChristoffel(nn.Module):
    """Gamma(v, v) = 20 tanh(((vU)^2 s) W^T / 20), s = 1/(1 + |vU| + 1e-6),
    plus the friction gate mu = 5 sigmoid(forget_gate(x) + input_gate(F)).

    Parameters and init follow gfn/geometry/lowrank.py:19-54.
    """

    def __init__(self, dim, rank=16, physics_config=None):
        super().__init__()
        self.dim = dim
        self.rank = rank
        self.config = physics_config or {}
        self.clamp_val = self.config.get("stability", {}).get("curvature_clamp", 5.0)
        self.is_torus = self.config.get("topology", {}).get("type", "").lower() == "torus"
        gate_input_dim = 2 * dim if self.is_torus else dim
        self.U = nn.Parameter(torch.zeros(dim, rank))
        self.W = nn.Parameter(torch.zeros(dim, rank))
        self.friction = self.config.get("stability", {}).get("friction", 0.05)
        self.V = nn.Linear(gate_input_dim, 1, bias=False)
        nn.init.zeros_(self.V.weight)
        self.gate_proj = nn.Linear(gate_input_dim, dim)
        nn.init.zeros_(self.gate_proj.weight)
        nn.init.constant_(self.gate_proj.bias, 2.0)
        self.forget_gate = nn.Linear(gate_input_dim, dim)
        nn.init.normal_(self.forget_gate.weight, std=0.01)
        self.input_gate = nn.Linear(dim, dim, bias=False)
        nn.init.normal_(self.input_gate.weight, std=0.01)
        nn.init.constant_(self.forget_gate.bias, 0.0)

    def forward(self, v, x=None, force=None, **kwargs):
        """Reference semantics gfn/geometry/lowrank.py:56-131 (CUDA tensors only)."""
        if self.is_torus:
            raise GfnError("toroidal Christoffel is not implemented on this build")
        require_cuda(v, x, force)
        gamma = ops.christoffel_fused(v, self.U, self.W)
        if x is None:
            return gamma
        Wf = kwargs.get("W_forget_stack", None)
        Wi = kwargs.get("W_input_stack", None)
        bf = kwargs.get("b_forget_stack", None)
        if Wf is not None and bf is not None:
            Wf = Wf[0] if Wf.dim() == 3 else Wf
            bf = bf[0] if bf.dim() == 2 else bf
            gate = torch.matmul(x, Wf.t()) + bf
            if Wi is not None and force is not None:
                Wi = Wi[0] if Wi.dim() == 3 else Wi
                gate = gate + torch.matmul(force, Wi.t())
        else:
            gate = self.forget_gate(x)
            if force is not None:
                gate = gate + self.input_gate(force)
        mu = torch.sigmoid(gate) * 5.0
        if getattr(self, "return_friction_separately", False):
            return gamma, mu
        # The combined form clamps gamma + mu v (lowrank.py:129-131); only the
        # non-leapfrog integrators use it.
        raise GfnError("combined Gamma + friction form is used only by the non-leapfrog "
                       "integrators, which this build does not implement")


class ReactiveChristoffel(LowRankChristoffel):
    """Active-inference wrapper (gfn/geometry/reactive.py:5-81).  With
    active_inference disabled (the configuration on the leapfrog path) it is
    exactly LowRankChristoffel."""

    def __init__(self, dim, rank=16, physics_config=None):
        super().__init__(dim, rank, physics_config=physics_config)
        self.config = physics_config or {}
        self.active_cfg = self.config.get("active_inference", {})
        self.plasticity = self.active_cfg.get("reactive_curvature", {}).get("plasticity", 0.0)
        self.singularity_threshold = self.active_cfg.get("singularities", {}).get("threshold", 0.8)
        self.black_hole_strength = self.active_cfg.get("singularities", {}).get("strength", 10.0)

    def forward(self, v, x=None, force=None, **kwargs):
        if self.active_cfg.get("enabled", False):
            raise GfnError("active-inference Christoffel (plasticity/singularities) is not "
                           "implemented on this build")
        return super().forward(v, x, force=force, **kwargs)


class ToroidalChristoffel(nn.Module):
    """Toroidal geometry (mirror of gfn/geometry/toroidal.py:4-148).

    Coordinates pair up as (theta, phi) = (x_i, x_i+1):
    Gamma_i = 0.05 (R + r cos th) sin th / r * v_ph^2,
    Gamma_i+1 = 0.05 * 2 (-(r sin th) / max(R + r cos th, 1e-6)) v_ph v_th;
    friction mu = 5 sigmoid(forget_gate([sin x, cos x]) + input_gate(F)).
    Parameters and init follow toroidal.py:17-52 (state_dict compatible).
    """

    def __init__(self, dim, physics_config=None):
        super().__init__()
        self.dim = dim
        self.config = physics_config or {}
        self.R = self.config.get("topology", {}).get("major_radius", 2.0)
        self.r = self.config.get("topology", {}).get("minor_radius", 1.0)
        self.topology_id = 1
        self.is_torus = True
        gate_input_dim = 2 * dim
        self.forget_gate = nn.Linear(gate_input_dim, dim)
        nn.init.normal_(self.forget_gate.weight, std=0.01)
        nn.init.constant_(self.forget_gate.bias, -5.0)
        self.input_gate = nn.Linear(dim, dim, bias=False)
        nn.init.normal_(self.input_gate.weight, std=0.01)
        self.clamp_val = self.config.get("stability", {}).get("curvature_clamp", 5.0)
        self.active_cfg = self.config.get("active_inference", {})
        self.plasticity = self.active_cfg.get("reactive_curvature", {}).get("plasticity", 0.1)
        self.singularity_threshold = self.active_cfg.get("singularities", {}).get("threshold", 0.8)
        self.black_hole_strength = self.active_cfg.get("singularities", {}).get("strength", 10.0)
        self.V = (nn.Linear(gate_input_dim, 1)
                  if self.active_cfg.get("singularities", {}).get("enabled", False) else None)
        if self.V is not None:
            nn.init.constant_(self.V.bias, -2.0)

    def forward(self, v, x=None, force=None, **kwargs):
        """Reference semantics gfn/geometry/toroidal.py:70-148 (CUDA tensors only)."""
        if x is None:
            return torch.zeros_like(v)
        if self.active_cfg.get("enabled", False):
            raise GfnError("active-inference toroidal Christoffel is not implemented on this build")
        require_cuda(v, x, force)
        gamma = ops.christoffel_fused(v, None, None, x, topology=1, R=self.R, r=self.r)
        x_in = torch.cat([torch.sin(x), torch.cos(x)], dim=-1)
        gate = self.forget_gate(x_in)
        if force is not None:
            gate = gate + self.input_gate(force)
        mu = torch.sigmoid(gate) * 5.0
        if getattr(self, "return_friction_separately", False):
            return gamma, mu
        return gamma + mu * v
