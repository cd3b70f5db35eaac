"""M-Layer and the parallel (scan) layer, mirrors of gfn/layers/base.py,
gfn/layers/parallel.py and gfn/layers/gating.py on the B200 kernels.

MLayer keeps the reference's submodule tree (christoffels, gatings,
friction_gates, integrators, out_proj_*, mixed_norm_*, norm_*) and its
construction order, so the same seed gives the same initial weights and a
reference state_dict loads as is.  Its forward runs one layer step of the
fused recurrence kernel.
"""
import torch
import torch.nn as nn

from ._lib import GfnError, require_cuda
from .cuda import ops
from .geometry import ReactiveChristoffel, ToroidalChristoffel
from .integrators import INTEGRATOR_CLASSES, SymplecticIntegrator
from .packing import PackCache


class RiemannianGating(nn.Module):
    """Curvature-based dt gate (gfn/layers/gating.py:4-51).  Parameters only:
    the dynamic-time option that uses it is off on the leapfrog path."""

    def __init__(self, dim, topology=0):
        super().__init__()
        self.topology = topology
        input_dim = 2 * dim if topology == 1 else dim
        self.curvature_net = nn.Sequential(nn.Linear(input_dim, dim // 4), nn.Tanh(),
                                           nn.Linear(dim // 4, 1), nn.Sigmoid())
        with torch.no_grad():
            nn.init.constant_(self.curvature_net[2].bias, 2.0)
            nn.init.xavier_uniform_(self.curvature_net[0].weight, gain=0.1)
            nn.init.xavier_uniform_(self.curvature_net[2].weight, gain=0.1)

    def forward(self, x):
        if self.topology == 1:
            x = torch.cat([torch.sin(x), torch.cos(x)], dim=-1)
        return self.curvature_net(x)


def _check_config(physics_config, integrator_type):
    pc = physics_config or {}
    if integrator_type in ("coupling", "neural"):
        raise GfnError(f"integrator_type={integrator_type!r} (a learned flow) is not implemented on "
                       "this build")
    for key in ("mixture", "hyper_curvature"):
        if pc.get(key, {}).get("enabled", False):
            raise GfnError(f"physics_config[{key!r}] is not implemented on this build")
    ai = pc.get("active_inference", {})
    torus = pc.get("topology", {}).get("type", "euclidean").lower() == "torus"
    if (integrator_type == "leapfrog" and not torus and ai.get("enabled", False)
            and (ai.get("reactive_curvature", {}).get("enabled", False)
                 or ai.get("singularities", {}).get("enabled", False))):
        # ReactiveChristoffel multiplies the (gamma, mu) pair the leapfrog asks
        # for by a tensor (gfn/geometry/reactive.py:54-72 after
        # gfn/integrators/symplectic/leapfrog.py:58): the reference fails here
        raise GfnError("reactive curvature / singularities with the Euclidean leapfrog: the "
                       "reference raises on this combination (tuple times tensor)")
    if pc.get("symmetries", {}).get("isomeric_groups"):
        raise GfnError("isomeric head groups are not implemented on this build")


# batch * dim from which the layer-by-layer path is faster than the fused
# persistent kernel (measured on B200: C3 256 x 512 and C4 4096 x 1024 are
# faster layered, C1 / C2 fused)
LAYERED_MIN_ELEMS = 1 << 17


def use_layered_path(path, heads, dim, batch):
    """True when the layer-by-layer (head-step kernel + tensor-core mixing
    GEMM) path computes the recurrence: `path` "layered", or "auto" with
    head mixing, a supported head dim and batch * dim >= LAYERED_MIN_ELEMS."""
    if heads == 1 or path == "fused":
        return False
    if path == "layered":
        return True
    return dim // heads in (16, 32, 64, 128) and batch * dim >= LAYERED_MIN_ELEMS


class MLayer(nn.Module):
    """One M-Layer: per-head leapfrog, head mixing, RMSNorm, saturation.

    Parameters/init: gfn/layers/base.py:34-196.  forward: base.py:198-338.
    """

    def __init__(self, dim, heads=4, rank=16, base_dt=0.1, integrator_type="heun",
                 physics_config=None, layer_idx=0, total_depth=6):
        super().__init__()
        assert dim % heads == 0, f"Dim {dim} must be divisible by heads {heads}"
        _check_config(physics_config, integrator_type)
        self.dim = dim
        self.heads = heads
        self.head_dim = dim // heads
        self.physics_config = physics_config or {}
        self.base_dt = self.physics_config.get("stability", {}).get("base_dt", base_dt)
        self.layer_idx = layer_idx
        self.total_depth = total_depth
        self.depth_scale = 1.0 / (total_depth ** 0.5)
        self.norm_x = nn.LayerNorm(dim)
        self.norm_v = nn.LayerNorm(dim)
        head_rank = max(4, rank // heads)
        topo_type = self.physics_config.get("topology", {}).get("type", "euclidean").lower()
        self.topology_id = 1 if topo_type == "torus" else 0
        Geo = ToroidalChristoffel if self.topology_id == 1 else ReactiveChristoffel
        self.christoffels = nn.ModuleList(
            [Geo(self.head_dim, physics_config=self.physics_config) if self.topology_id == 1
             else Geo(self.head_dim, head_rank, physics_config=self.physics_config)
             for _ in range(heads)])
        self.register_buffer("headless_mode", torch.tensor(False))
        self.use_dynamic_time = self.physics_config.get("active_inference", {}).get("dynamic_time", {}).get("enabled", False)
        self.gatings = nn.ModuleList([RiemannianGating(self.head_dim, topology=self.topology_id)
                                      for _ in range(heads)])
        scale_vals = []
        for i in range(heads):
            target_dt = self.base_dt / 0.9
            val_init = torch.tensor(target_dt).exp().sub(1.0).log()
            scale_vals.append(val_init + i * 0.1)
        self.dt_params = nn.Parameter(torch.tensor(scale_vals))
        self.time_heads = None
        self.friction_gates = nn.ModuleList([self.christoffels[i].forget_gate for i in range(heads)])
        Integ = INTEGRATOR_CLASSES.get(integrator_type, SymplecticIntegrator)
        self.integrator_type = integrator_type
        self.integrators = nn.ModuleList([Integ(self.christoffels[i], dt=self.base_dt) for i in range(heads)])
        # the fused / layered recurrence kernels compute the Euclidean
        # leapfrog; every other configuration steps layer by layer through the
        # multi-scheme integrator kernel (generic path)
        ai = self.physics_config.get("active_inference", {})
        self.use_dynamic_time = ai.get("dynamic_time", {}).get("enabled", False)
        self.generic = (self.topology_id == 1 or integrator_type != "leapfrog" or self.use_dynamic_time
                        or ai.get("recursive_geodesics", {}).get("enabled", False)
                        or (ai.get("enabled", False)
                            and (ai.get("reactive_curvature", {}).get("enabled", False)
                                 or ai.get("singularities", {}).get("enabled", False))))
        if heads > 1:
            self.out_proj_x = nn.Linear(3 * dim if self.topology_id == 1 else dim, dim)
            self.out_proj_v = nn.Linear(dim, dim)
            self.mixed_norm_x = nn.RMSNorm(dim)
            self.mixed_norm_v = nn.RMSNorm(dim)
            nn.init.xavier_uniform_(self.out_proj_x.weight)
            nn.init.zeros_(self.out_proj_x.bias)
            nn.init.xavier_uniform_(self.out_proj_v.weight)
            nn.init.zeros_(self.out_proj_v.bias)
        self.use_recursive = ai.get("recursive_geodesics", {}).get("enabled", False)
        if self.use_recursive:
            self.context_proj = nn.Linear(heads, dim)
            nn.init.zeros_(self.context_proj.weight)
        self._pack = PackCache()
        # "auto" (by batch size), "fused" or "layered": which recurrence kernel
        # computes an inference step (the same choice as Manifold.recurrence)
        self.recurrence_path = "auto"

    def forward(self, x, v, force=None, context=None, collect_christ=False):
        """One layer step for every row: returns (x_next, v_next, context, [])."""
        require_cuda(x, v, force)
        if collect_christ:
            raise GfnError("collect_christ is not supported by the fused kernels")
        B = x.shape[0]
        if force is None:
            force = torch.zeros_like(x)
        if self.generic or (self.training_generic() and self.training and torch.is_grad_enabled()):
            return self._generic_step(x, v, force, context)
        if torch.is_grad_enabled() and any(t.requires_grad for t in
                                           [x, v, force, *self.parameters()]):
            from .training import leapfrog_sequence_train
            _, _, xn, vn = leapfrog_sequence_train([self], x, v, force.reshape(B, 1, self.dim))
            return xn, vn, torch.ones(B, self.heads, device=x.device, dtype=x.dtype), []
        layered = use_layered_path(self.recurrence_path, self.heads, self.dim, B)
        packed, meta = self._pack.get([self], layered=layered)
        seq = ops.leapfrog_layered_sequence if layered else ops.leapfrog_sequence
        _, _, xn, vn = seq(x, v, packed, meta, self.base_dt, forces=force.reshape(B, 1, self.dim),
                           want_x_seq=False, want_v_seq=False)
        context_next = torch.ones(B, self.heads, device=x.device, dtype=x.dtype)
        return xn, vn, context_next, []

    def training_generic(self):
        """True when training takes the generic layer step: the generic
        configurations, and head dims above the fused BPTT kernels' 64 (the
        per-head leapfrog autograd operator takes up to 256)."""
        return self.generic or self.head_dim > 64

    def _generic_step(self, x, v, force, context=None):
        """One layer step for the torus and the non-leapfrog integrators:
        every head's integrator in one launch of the multi-scheme kernel, then
        the head mixing of gfn/layers/base.py:304-335 (torus: the mixer reads
        [sin x, cos x, tanh(v / 100)] and x wraps into [0, 2 pi) instead of
        the RMSNorm)."""
        if self.training and torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()):
            ai = self.physics_config.get("active_inference", {})
            if (self.integrator_type != "leapfrog" or self.use_dynamic_time
                    or (ai.get("enabled", False) and (ai.get("reactive_curvature", {}).get("enabled", False)
                                                      or ai.get("singularities", {}).get("enabled", False)))):
                return self._generic_step_train_scheme(x, v, force, context)
            return self._generic_step_train(x, v, force, context)
        with torch.no_grad():
            return self._generic_step_nograd(x, v, force, context)

    def _generic_step_train(self, x, v, force, context):
        """Differentiable leapfrog layer step for the torus (and the Euclidean
        leapfrog with recursive geodesics): per head the leapfrog autograd
        operator (forward kernel, reverse-replay backward with the gradients of
        the state, force, U, W, the forget gate and the dt scale), then the
        head mixing of gfn/layers/base.py:304-335 with torch's autograd."""
        B = x.shape[0]
        H, hd = self.heads, self.head_dim
        if self.use_recursive and context is not None:
            force = force + self.context_proj(context)
        dts = torch.nn.functional.softplus(self.dt_params)
        xo, vo = [], []
        for h, ch in enumerate(self.christoffels):
            sl = slice(h * hd, (h + 1) * hd)
            if self.topology_id == 1:
                U = W = None
                R, r = ch.R, ch.r
            else:
                U, W, R, r = ch.U, ch.W, 2.0, 1.0
            xh, vh = ops.leapfrog_fused(x[:, sl].contiguous(), v[:, sl].contiguous(), force[:, sl].contiguous(),
                                        U, W, self.base_dt, dts[h:h + 1], 1, topology=self.topology_id,
                                        Wf=ch.forget_gate.weight, bf=ch.forget_gate.bias, R=R, r=r)
            xo.append(xh)
            vo.append(vh)
        xc, vc = torch.cat(xo, -1), torch.cat(vo, -1)
        return self._mix(xc, vc, B, H)

    def _generic_step_train_scheme(self, x, v, force, context):
        """Differentiable layer step for the non-leapfrog integrators, dynamic
        time and the active curvature terms: the same scheme arithmetic as the
        multi-scheme kernel (gfn/integrators/**), on [B, H, hd] tensors for all
        heads at once through torch's autograd (inference uses the kernel)."""
        from .integrators import scheme_step_torch
        B = x.shape[0]
        H, hd = self.heads, self.head_dim
        if self.use_recursive and context is not None:
            force = force + self.context_proj(context)
        ch = self.christoffels
        Wf = torch.stack([c.forget_gate.weight for c in ch])
        bf = torch.stack([c.forget_gate.bias for c in ch])
        Wi = torch.stack([c.input_gate.weight for c in ch])
        if self.topology_id == 0:
            U = torch.stack([c.U for c in ch])
            W = torch.stack([c.W for c in ch])
            R = r = 1.0
        else:
            U = W = None
            R, r = ch[0].R, ch[0].r
        dts = torch.nn.functional.softplus(self.dt_params).view(1, H, 1)
        gates = None
        if self.use_dynamic_time:
            # dt scale per head and row (gfn/layers/base.py:219-229)
            hv = x.view(B, H, hd)
            gates = torch.stack([self.gatings[i](hv[:, i]) for i in range(H)], dim=0)  # [H, B, 1]
            dts = dts.view(H, 1, 1) * gates                                           # [H, B, 1]
            dts = dts.permute(1, 0, 2)                                                # [B, H, 1]
        scheme = self.integrator_type if self.integrator_type in ops.SCHEMES else "verlet"
        plast, mode, V, Vb, thr, strength = self._active_terms()
        act = None
        if plast or mode:
            act = dict(plasticity=plast, V=V, Vb=Vb, thr=thr, strength=strength)
        leap = scheme == "leapfrog"
        xh, vh = scheme_step_torch(scheme, x.reshape(B, H, hd), v.reshape(B, H, hd), force.reshape(B, H, hd),
                                   U, W, Wf, bf, None if leap else Wi, self.base_dt * dts, self.topology_id, R, r,
                                   act)
        xn, vn, ctx, _ = self._mix(xh.reshape(B, H * hd), vh.reshape(B, H * hd), B, H)
        if gates is not None:
            ctx = gates.squeeze(-1).t()
        return xn, vn, ctx, []

    def _mix(self, xc, vc, B, H):
        if H > 1:
            if self.topology_id == 1:
                mix_in = torch.cat([torch.sin(xc), torch.cos(xc), torch.tanh(vc / 100.0)], dim=-1)
                xn = torch.remainder(self.out_proj_x(mix_in), 2.0 * 3.14159265359)
            else:
                xn = self.mixed_norm_x(self.out_proj_x(xc))
            vn = self.mixed_norm_v(self.out_proj_v(vc))
        else:
            xn, vn = xc, vc
        vn = 100.0 * torch.tanh(vn / 100.0)
        return xn, vn, torch.ones(B, H, device=xc.device, dtype=xc.dtype), []

    def _active_terms(self):
        """Active-inference operands (gfn/geometry/reactive.py:53-81,
        gfn/geometry/toroidal.py:126-141): plasticity, singularity mode,
        potential weights / bias, threshold, strength."""
        ai = self.physics_config.get("active_inference", {})
        ch = self.christoffels
        if not ai.get("enabled", False):
            return 0.0, 0, None, None, 1.0, 1.0
        plast = ch[0].plasticity if ai.get("reactive_curvature", {}).get("enabled", False) else 0.0
        mode, V, Vb = 0, None, None
        if ai.get("singularities", {}).get("enabled", False) and getattr(ch[0], "V", None) is not None:
            mode = 2 if self.topology_id == 1 else 1
            V = torch.stack([c.V.weight.reshape(-1) for c in ch]).contiguous()
            if ch[0].V.bias is not None:
                Vb = torch.stack([c.V.bias.reshape(()) for c in ch]).contiguous()
        return (float(plast), mode, V, Vb, float(ch[0].singularity_threshold),
                float(ch[0].black_hole_strength))

    def _generic_step_nograd(self, x, v, force, context):
        B = x.shape[0]
        if self.use_recursive and context is not None:
            force = force + self.context_proj(context)
        H, hd = self.heads, self.head_dim
        leap = self.integrator_type == "leapfrog"
        ch = self.christoffels
        Wf = torch.stack([c.forget_gate.weight for c in ch]).contiguous()
        bf = torch.stack([c.forget_gate.bias for c in ch]).contiguous()
        Wi = None if leap else torch.stack([c.input_gate.weight for c in ch]).contiguous()
        if self.topology_id == 0:
            U = torch.stack([c.U for c in ch]).contiguous()
            W = torch.stack([c.W for c in ch]).contiguous()
            R = r = 1.0
        else:
            U = W = None
            R, r = ch[0].R, ch[0].r
        scheme = self.integrator_type if self.integrator_type in ops.SCHEMES else "verlet"
        dt_base = torch.nn.functional.softplus(self.dt_params)
        if self.use_dynamic_time:
            # dt scale per head and row: softplus(dt_params) * curvature gate
            # (gfn/layers/base.py:219-229, gfn/layers/gating.py:38-51)
            hv = x.view(B, H, hd)
            gates = torch.stack([self.gatings[i](hv[:, i]) for i in range(H)], dim=0)  # [H, B, 1]
            dts = (dt_base.view(H, 1, 1) * gates).squeeze(-1).t().contiguous()       # [B, H]
            if H == 1:
                dts = dts.reshape(B)
            context_next = gates.squeeze(-1).t()
        else:
            dts = dt_base
            context_next = torch.ones(B, H, device=x.device, dtype=x.dtype)
        plast, mode, V, Vb, thr, strength = self._active_terms()
        xc, vc = ops.integrator_heads(scheme, x.contiguous(), v.contiguous(), force.contiguous(), U, W,
                                      self.base_dt, dts, 1, self.topology_id, Wf, bf, Wi, H, R, r,
                                      plast, V, Vb, mode, thr, strength)
        if H > 1:
            if self.topology_id == 1:
                mix_in = torch.cat([torch.sin(xc), torch.cos(xc), torch.tanh(vc / 100.0)], dim=-1)
                xn = torch.remainder(self.out_proj_x(mix_in), 2.0 * 3.14159265359)
            else:
                xn = self.mixed_norm_x(self.out_proj_x(xc))
            vn = self.mixed_norm_v(self.out_proj_v(vc))
        else:
            xn, vn = xc, vc
        vn = 100.0 * torch.tanh(vn / 100.0)
        return xn, vn, context_next, []


class ParallelMLayer(nn.Module):
    """Linearised layer for the scan path (gfn/layers/parallel.py:5-125):
    force -> LayerNorm -> A = sigmoid(to_A), dt = softplus(to_dt) * 0.1 * 1.5^head,
    B = to_B * dt -> v = scan(A, B), x = scan(1, v dt).

    The three projections run as one split-fp16 tensor-core GEMM against the
    concatenated weight (`split_gemm = False`: torch's fp32 matmul); the two
    scans and all elementwise work run in one fused kernel.
    """

    def __init__(self, dim, heads=4, physics_config=None, **kwargs):
        super().__init__()
        assert dim % heads == 0
        self.dim = dim
        self.heads = heads
        self.head_dim = dim // heads
        self.norm_x = nn.LayerNorm(dim)
        self.norm_v = nn.LayerNorm(dim)
        self.to_A = nn.Sequential(nn.Linear(dim, dim), nn.Sigmoid())
        self.to_B = nn.Linear(dim, dim)
        self.to_dt = nn.Sequential(nn.Linear(dim, dim), nn.Softplus())
        scale_vec = []
        for i in range(heads):
            scale_vec.extend([1.5 ** i] * (dim // heads))
        self.register_buffer("base_dt_scales", torch.tensor(scale_vec, dtype=torch.float32))
        self.base_dt = 0.1
        if heads > 1:
            self.out_proj = nn.Linear(dim * 2, dim * 2)
        # True: the projections on the tensor cores (split fp16); False: torch's fp32 matmul
        self.split_gemm = True

    def forward(self, x, v, force, collect_christ=False):
        require_cuda(force)
        if x is not None:
            raise GfnError("ParallelMLayer with an explicit x is not used by the reference model")
        f = self.norm_x(force)
        Wcat = torch.cat([self.to_A[0].weight, self.to_dt[0].weight, self.to_B.weight], 0)
        bcat = torch.cat([self.to_A[0].bias, self.to_dt[0].bias, self.to_B.bias], 0)
        if self.split_gemm and f.is_cuda:
            # the three projections as one tensor-core GEMM over split-fp16
            # operands (~1e-6 relative, float32-level; manifold_b200.readout)
            from .readout import SplitLinear
            B, L, _ = f.shape
            z = SplitLinear.apply(f.reshape(B * L, self.dim), Wcat, bcat).reshape(B, L, 3 * self.dim)
        else:
            z = torch.nn.functional.linear(f, Wcat, bcat)
        x_seq, v_seq = ops.parallel_layer_scan(z, self.heads, self.base_dt)
        return x_seq, v_seq, None, []
