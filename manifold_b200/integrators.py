"""Leapfrog (kick-drift-kick) integrator, mirror of
gfn/integrators/symplectic/leapfrog.py on the B200 kernels."""
import torch
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


def _gates(christoffel, force, kwargs, with_input):
    """The friction gate the reference's Christoffel applies: the forget /
    input stacks MLayer passes (gfn/geometry/lowrank.py:108-117; the torus
    reads its own gates, gfn/geometry/toroidal.py:113-124), else the module's
    own gates (lowrank.py:118-121).  Returns (Wf, bf, Wi)."""
    Wf = kwargs.get("W_forget_stack", None)
    Wi = kwargs.get("W_input_stack", None)
    bf = kwargs.get("b_forget_stack", None)
    if getattr(christoffel, "is_torus", False) or Wf is None or bf is None:
        gate = getattr(christoffel, "forget_gate", None)
        if gate is None:
            return None, None, None
        ig = getattr(christoffel, "input_gate", None)
        Wi = ig.weight if (ig is not None and force is not None and with_input) else None
        return gate.weight, gate.bias, Wi
    Wf = Wf[0] if Wf.dim() == 3 else Wf
    bf = bf[0] if bf.dim() == 2 else bf
    if Wi is not None and Wi.dim() == 3:
        Wi = Wi[0]
    if force is None or not with_input:
        Wi = None
    return Wf, bf, Wi


class _SchemeIntegrator(nn.Module):
    """Base of the non-leapfrog integrators: forward(x, v, force, dt_scale,
    steps) -> (x, v) through the library's multi-scheme kernel, with the
    acceleration a = F - Christoffel(v, x, F) in the Christoffel's combined
    form (friction included)."""

    scheme = None

    def __init__(self, christoffel, dt=0.01):
        super().__init__()
        self.christoffel = christoffel
        self.dt = dt

    def forward(self, x, v, force=None, dt_scale=1.0, steps=1, collect_christ=False, **kwargs):
        require_cuda(x, v, force)
        topology = 1 if getattr(self.christoffel, "is_torus", False) else 0
        Wf, bf, Wi = _gates(self.christoffel, force, kwargs, True)
        U = getattr(self.christoffel, "U", None)
        W = getattr(self.christoffel, "W", None)
        if topology == 0 and (U is None or W is None):
            raise GfnError(f"{type(self).__name__} needs a low-rank Christoffel (U, W) or the torus")
        return ops.integrator_heads(self.scheme, x, v, force, U, W, self.dt, dt_scale, steps, topology,
                                    Wf, bf, Wi, 1, getattr(self.christoffel, "R", 2.0),
                                    getattr(self.christoffel, "r", 1.0))


class EulerIntegrator(_SchemeIntegrator):
    """gfn/integrators/runge_kutta/euler.py:20-64."""
    scheme = "euler"


class HeunIntegrator(_SchemeIntegrator):
    """gfn/integrators/runge_kutta/heun.py:20-78 (the reference's default)."""
    scheme = "heun"


class RK4Integrator(_SchemeIntegrator):
    """gfn/integrators/runge_kutta/rk4.py:20-83."""
    scheme = "rk4"


class DormandPrinceIntegrator(_SchemeIntegrator):
    """gfn/integrators/runge_kutta/dormand_prince.py:20-122 (fixed step, 5th-order weights)."""
    scheme = "dormand_prince"


class SymplecticIntegrator(_SchemeIntegrator):
    """Velocity Verlet (gfn/integrators/symplectic/verlet.py:20-73)."""
    scheme = "verlet"


VerletIntegrator = SymplecticIntegrator


class YoshidaIntegrator(_SchemeIntegrator):
    """gfn/integrators/symplectic/yoshida.py:18-86."""
    scheme = "yoshida"


class ForestRuthIntegrator(_SchemeIntegrator):
    """gfn/integrators/symplectic/forest_ruth.py:20-89."""
    scheme = "forest_ruth"


class OmelyanIntegrator(_SchemeIntegrator):
    """gfn/integrators/symplectic/omelyan.py:18-96 (PEFRL)."""
    scheme = "omelyan"


INTEGRATOR_CLASSES = {
    "leapfrog": LeapfrogIntegrator, "euler": EulerIntegrator, "heun": HeunIntegrator,
    "rk4": RK4Integrator, "rk45": DormandPrinceIntegrator, "yoshida": YoshidaIntegrator,
    "forest_ruth": ForestRuthIntegrator, "omelyan": OmelyanIntegrator,
}


# ---------------------------------------------------------------- training form
# The scheme arithmetic of the multi-scheme kernel on [B, H, hd] tensors with
# torch's autograd: used by MLayer in training for the non-leapfrog
# integrators (inference runs the kernel).

def _active_factor_torch(x, v, act, topology):
    """The active-inference multiplier of the Christoffel term
    (gfn/geometry/reactive.py:62-81, gfn/geometry/toroidal.py:126-141)."""
    m = 1.0
    if act.get("plasticity", 0.0):
        m = m * (1.0 + act["plasticity"] * torch.tanh((v * v).mean(-1, keepdim=True)))
    if act.get("V") is not None:
        feat = torch.cat([torch.sin(x), torch.cos(x)], -1) if topology == 1 else x
        z = torch.einsum("bhk,hk->bh", feat, act["V"]).unsqueeze(-1)
        if act.get("Vb") is not None:
            z = z + act["Vb"].view(1, -1, 1)
        pot = torch.sigmoid(z)
        sg = (pot > act["thr"]).to(x.dtype) if topology == 1 else torch.sigmoid(10.0 * (pot - act["thr"]))
        m = m * (1.0 + sg * (act["strength"] - 1.0))
    return m


def _torus_gamma_torch(x, v, R, r):
    th, vth, vph = x[..., 0::2], v[..., 0::2], v[..., 1::2]
    denom = R + r * torch.cos(th)
    g0 = denom * torch.sin(th) / r * vph ** 2
    g1 = 2.0 * (-(r * torch.sin(th)) / torch.clamp(denom, min=1e-6)) * vph * vth
    return torch.stack([g0, g1], -1).reshape(x.shape) * 0.05


def _lowrank_pre_torch(v, U, W):
    p = torch.einsum("bhk,hkr->bhr", v, U)
    s = 1.0 / (1.0 + torch.norm(p, dim=-1, keepdim=True) + 1e-6)
    return torch.einsum("bhr,hkr->bhk", (p * p) * s, W)


def _mu_torch(x, F, Wf, bf, Wi, topology):
    feat = torch.cat([torch.sin(x), torch.cos(x)], -1) if topology == 1 else x
    gate = torch.einsum("bhk,hjk->bhj", feat, Wf) + bf
    if Wi is not None:
        gate = gate + torch.einsum("bhk,hjk->bhj", F, Wi)
    return torch.sigmoid(gate) * 5.0


def _accel_torch(x, v, F, U, W, Wf, bf, Wi, topology, R, r, act=None):
    """a = F - C(v, x), C the Christoffel term in its combined form
    (gfn/geometry/lowrank.py:100-131, gfn/geometry/toroidal.py:70-148)."""
    mu = _mu_torch(x, F, Wf, bf, Wi, topology)
    M = _active_factor_torch(x, v, act, topology) if act else 1.0
    if topology == 1:
        return F - (_torus_gamma_torch(x, v, R, r) * M + mu * v)
    pre = _lowrank_pre_torch(v, U, W)
    return F - 20.0 * torch.tanh((pre + mu * v) / 20.0) * M


def _wrap(x, topology):
    return torch.remainder(x, 2.0 * 3.14159265359) if topology == 1 else x


_CBRT2 = 2.0 ** (1.0 / 3.0)
_FR_TH = 1.0 / (2.0 - _CBRT2)
_SYMPLECTIC = {
    "yoshida": ([_FR_TH / 2, (1 - _FR_TH) / 2, (1 - _FR_TH) / 2, _FR_TH / 2],
                [_FR_TH, 1 - 2 * _FR_TH, _FR_TH, _FR_TH]),
    "omelyan": ([0.1786178958448091, -0.06626458266981849,
                 1.0 - 2.0 * (-0.06626458266981849 + 0.1786178958448091), -0.06626458266981849,
                 0.1786178958448091],
                [(1.0 + 2.0 * 0.2123418310626054) / 2.0, -0.2123418310626054, -0.2123418310626054,
                 (1.0 + 2.0 * 0.2123418310626054) / 2.0, (1.0 + 2.0 * 0.2123418310626054) / 2.0]),
}
_SYMPLECTIC["forest_ruth"] = _SYMPLECTIC["yoshida"]
_DP_A = [[1 / 5], [3 / 40, 9 / 40], [44 / 45, -56 / 15, 32 / 9],
         [19372 / 6561, -25360 / 2187, 64448 / 6561, -212 / 729],
         [9017 / 3168, -355 / 33, 46732 / 5247, 49 / 176, -5103 / 18656]]
_DP_B = [35 / 384, 0, 500 / 1113, 125 / 192, -2187 / 6784, 11 / 84]


def scheme_step_torch(scheme, x, v, F, U, W, Wf, bf, Wi, dt, topology=0, R=2.0, r=1.0, act=None):
    """One step of `scheme` (gfn/integrators/**) with a differentiable dt
    ([1, H, 1] or per row [B, H, 1]); act: the active-inference terms."""
    def acc(xx, vv):
        return _accel_torch(xx, vv, F, U, W, Wf, bf, Wi, topology, R, r, act)

    if scheme == "leapfrog":
        # implicit friction, forget gate only (gfn/integrators/symplectic/leapfrog.py:50-114)
        h = 0.5 * dt
        for half in range(2):
            mu = _mu_torch(x, F, Wf, bf, None, topology)
            g = (_torus_gamma_torch(x, v, R, r) if topology == 1
                 else 20.0 * torch.tanh(_lowrank_pre_torch(v, U, W) / 20.0))
            if act:
                g = g * _active_factor_torch(x, v, act, topology)
            v = (v + h * (F - g)) / (1.0 + h * mu)
            if half == 0:
                x = _wrap(x + dt * v, topology)
        return x, v

    if scheme == "euler":
        a = acc(x, v)
        return _wrap(x + dt * v, topology), v + dt * a
    if scheme == "heun":
        dv1 = acc(x, v)
        vp = v + dt * dv1
        xp = _wrap(x + dt * v, topology)
        dv2 = acc(xp, vp)
        return _wrap(x + (dt / 2.0) * (v + vp), topology), v + (dt / 2.0) * (dv1 + dv2)
    if scheme == "rk4":
        hh = 0.5 * dt
        dv1 = acc(x, v)
        v2, x2 = v + hh * dv1, _wrap(x + hh * v, topology)
        dv2 = acc(x2, v2)
        v3, x3 = v + hh * dv2, _wrap(x + hh * v2, topology)
        dv3 = acc(x3, v3)
        v4, x4 = v + dt * dv3, _wrap(x + dt * v3, topology)
        dv4 = acc(x4, v4)
        return (_wrap(x + (dt / 6.0) * (v + 2 * v2 + 2 * v3 + v4), topology),
                v + (dt / 6.0) * (dv1 + 2 * dv2 + 2 * dv3 + dv4))
    if scheme == "verlet":
        vh = v + 0.5 * dt * acc(x, v)
        x = _wrap(x + dt * vh, topology)
        return x, vh + 0.5 * dt * acc(x, vh)
    if scheme in _SYMPLECTIC:
        cs, ds = _SYMPLECTIC[scheme]
        for c, dd in zip(cs, ds):
            x = _wrap(x + c * dt * v, topology)
            v = v + dd * dt * acc(x, v)
        return x, v
    if scheme in ("rk45", "dormand_prince"):
        kx, kv = [v], [acc(x, v)]
        for row in _DP_A:
            sx = sum(a * kx[j] for j, a in enumerate(row))
            sv = sum(a * kv[j] for j, a in enumerate(row))
            xs, vs = _wrap(x + dt * sx, topology), v + dt * sv
            kx.append(vs)
            kv.append(acc(xs, vs))
        sx = sum(b * kx[j] for j, b in enumerate(_DP_B) if b)
        sv = sum(b * kv[j] for j, b in enumerate(_DP_B) if b)
        return _wrap(x + dt * sx, topology), v + dt * sv
    raise GfnError(f"scheme {scheme!r}")
