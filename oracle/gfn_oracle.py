"""CPU restatement (numpy) of the reference's recurrent geodesic-flow hot path.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
path: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import it.  The product (``manifold_b200``) never calls it;
there is no CPU fallback.

Every function restates the reference's PyTorch CPU code path (Manifold-
Laboratory/manifold, package ``gfn``) in numpy, in the dtype of its inputs
(float32 for parity, float64 for drift references), keeping the reference's
order of operations so that float32 results round the same way wherever the
reference does elementwise work.  Citations are ``gfn/<file>:<line>``.

Parity pin: the reference's own tests hold no golden vectors for this path,
so this restatement is pinned against fixtures produced by running the
reference itself (``tests/golden/make_golden.py`` imports ``gfn`` and records
its outputs on seeded inputs); ``tests/test_oracle_golden.py`` checks it.

Canonical parameter layout (numpy arrays), one dict per layer::

    U, W      [H, hd, r]    low-rank Christoffel factors   (gfn/geometry/lowrank.py:31-32)
    Wf        [H, hd, hd]   forget_gate.weight, [out, in]  (gfn/geometry/lowrank.py:47)
    bf        [H, hd]       forget_gate.bias
    dt_params [H]           raw per-head dt parameters     (gfn/layers/base.py:132-139)
    Wx, Wv    [d, d]        out_proj_{x,v}.weight, [out,in] (gfn/layers/base.py:181-182)
    bx, bv    [d]           out_proj_{x,v}.bias
    gx, gv    [d]           mixed_norm_{x,v}.weight        (gfn/layers/base.py:185-186)
"""
import numpy as np

# torch.finfo(torch.float32).eps -- nn.RMSNorm(eps=None) uses the input
# dtype's machine epsilon (gfn/layers/base.py:185-186).
def _rms_eps(dtype):
    return np.finfo(dtype).eps


def softplus(x):
    """torch.nn.functional.softplus with beta=1, threshold=20."""
    x = np.asarray(x)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(x.dtype)


def sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(x.dtype)


def christoffel(v, U, W):
    """Low-rank Christoffel contraction Gamma(v, v).

    gfn/geometry/lowrank.py:93-98 (proj, norm, scale, sq, gamma) and the soft
    clamp 20*tanh(gamma/20) applied when friction is returned separately
    (gfn/geometry/lowrank.py:125-127).  v: [B, hd]; U, W: [hd, r].
    """
    dt = v.dtype
    one = dt.type(1.0)
    proj = v @ U                                              # [B, r]
    norm = np.sqrt(np.sum(proj * proj, axis=-1, keepdims=True))
    scale = one / ((one + norm) + dt.type(1e-6))
    sq = (proj * proj) * scale
    gamma = sq @ W.T                                          # [B, hd]
    return dt.type(20.0) * np.tanh(gamma / dt.type(20.0))


def friction(x, Wf, bf):
    """mu = 5 * sigmoid(x Wf^T + bf)  (gfn/integrators/symplectic/leapfrog.py:72-81)."""
    gate = (x @ Wf.T) + bf
    return sigmoid(gate) * x.dtype.type(5.0)


def leapfrog_head_step(x, v, F, U, W, Wf, bf, dt, dt_scale, steps=1):
    """One head's kick-drift-kick with implicit friction.

    gfn/integrators/symplectic/leapfrog.py:50-114 (steps loop, h = dt*scale/2,
    v_half = (v + h(F - G(v)))/(1 + h mu(x)), x += dt_eff v_half,
    v = (v_half + h(F - G(v_half)))/(1 + h mu(x'))).  Euclidean boundary is
    the identity (gfn/geometry/boundaries.py:4-17).
    """
    dtp = x.dtype.type
    eff = dtp(dt) * dtp(dt_scale)
    h = dtp(0.5) * eff
    one = dtp(1.0)
    for _ in range(steps):
        g0 = christoffel(v, U, W)
        mu0 = friction(x, Wf, bf)
        v_half = (v + h * (F - g0)) / (one + h * mu0)
        x = x + eff * v_half
        g1 = christoffel(v_half, U, W)
        mu1 = friction(x, Wf, bf)
        v = (v_half + h * (F - g1)) / (one + h * mu1)
    return x, v


TWO_PI_F32 = np.float32(2.0 * 3.14159265359)  # gfn/geometry/boundaries.py:13-14


def torus_wrap(x):
    """torch.remainder(x, 2*PI) (gfn/geometry/boundaries.py:4-17): fmod, then
    shifted into [0, 2 pi) for negative remainders."""
    m = np.fmod(x, x.dtype.type(TWO_PI_F32))
    return np.where(m < 0, m + x.dtype.type(TWO_PI_F32), m).astype(x.dtype)


def torus_christoffel(v, x, R=2.0, r=1.0):
    """Toroidal Gamma (gfn/geometry/toroidal.py:70-108): for pairs
    (th, ph) = (x_i, x_i+1), Gamma_i = (R + r cos th) sin th / r * v_ph^2,
    Gamma_i+1 = 2 (-(r sin th) / max(R + r cos th, 1e-6)) v_ph v_th, times 0.05."""
    dt = v.dtype.type
    g = np.zeros_like(v)
    R, r = dt(R), dt(r)
    for i in range(0, v.shape[-1] - 1, 2):
        th, vth, vph = x[..., i], v[..., i], v[..., i + 1]
        denom = R + r * np.cos(th)
        ds = np.maximum(denom, dt(1e-6))
        g[..., i] = (denom * np.sin(th) / r) * (vph ** 2)
        g[..., i + 1] = dt(2.0) * (-(r * np.sin(th)) / ds) * vph * vth
    return g * dt(0.05)


def leapfrog_head_step_gated(x, v, F, U, W, Wf, bf, Wi, dt, dt_scale, steps=1, topology=0,
                             R=2.0, r=1.0, act=None):
    """leapfrog_head_step with the full friction gate and both topologies:
    mu = 5 sigmoid((feat(x) Wf^T + bf) + F Wi^T) (gfn/geometry/lowrank.py:114-123;
    Wi None: no input gate), feat = [sin x, cos x] and Gamma the toroidal term
    on the torus (gfn/geometry/toroidal.py:70-124), x wrapped after the drift
    (gfn/integrators/symplectic/leapfrog.py:88-91)."""
    dtp = x.dtype.type
    eff = dtp(dt) * dtp(dt_scale)
    h = dtp(0.5) * eff
    one = dtp(1.0)
    zin = (F @ Wi.T) if Wi is not None else dtp(0.0)

    def mu(xc):
        if Wf is None:
            return dtp(0.0)
        feat = np.concatenate([np.sin(xc), np.cos(xc)], -1) if topology == 1 else xc
        return sigmoid(((feat @ Wf.T) + bf) + zin) * dtp(5.0)

    def gam(vc, xc):
        g = torus_christoffel(vc, xc, R, r) if topology == 1 else christoffel(vc, U, W)
        return g * active_factor(xc, vc, act, topology) if act is not None else g

    for _ in range(steps):
        v_half = (v + h * (F - gam(v, x))) / (one + h * mu(x))
        x = x + eff * v_half
        if topology == 1:
            x = torus_wrap(x)
        v = (v_half + h * (F - gam(v_half, x))) / (one + h * mu(x))
    return x, v


def active_factor(x, v, act, topology):
    """Active-inference multiplier of the Christoffel term (gfn/geometry/reactive.py:62-81,
    gfn/geometry/toroidal.py:126-141): (1 + plasticity tanh(mean v^2)) times
    (1 + s (strength - 1)), s = sigmoid(10 (p - thr)) (low-rank) or [p > thr]
    (torus), p = sigmoid(feat(x) . V + b).  act None: 1."""
    dtp = x.dtype.type
    if act is None:
        return dtp(1.0)
    m = dtp(1.0)
    if act.get("plasticity", 0.0):
        energy = np.tanh(np.mean(v * v, axis=-1, keepdims=True))
        m = m * (dtp(1.0) + dtp(act["plasticity"]) * energy)
    if act.get("V") is not None:
        feat = np.concatenate([np.sin(x), np.cos(x)], -1) if topology == 1 else x
        z = feat @ act["V"][:, None]
        if act.get("Vb") is not None:
            z = z + act["Vb"]
        pot = sigmoid(z.astype(x.dtype))
        if topology == 1:
            sg = (pot > dtp(act["thr"])).astype(x.dtype)
        else:
            sg = sigmoid((dtp(10.0) * (pot - dtp(act["thr"]))).astype(x.dtype))
        m = m * (dtp(1.0) + sg * (dtp(act["strength"]) - dtp(1.0)))
    return m


def combined_accel(x, v, F, U, W, Wf, bf, Wi, topology=0, R=2.0, r=1.0, act=None):
    """a = F - C(v, x): the Christoffel term in the combined form the
    non-leapfrog integrators call (gfn/geometry/lowrank.py:100-131,
    gfn/geometry/toroidal.py:70-148): mu = 5 sigmoid(feat(x) Wf^T + bf + F Wi^T);
    low-rank C = 20 tanh((((vU)^2 s) W^T + mu v) / 20), torus C = Gamma + mu v."""
    dtp = x.dtype.type
    if Wf is not None:
        feat = np.concatenate([np.sin(x), np.cos(x)], -1) if topology == 1 else x
        gate = (feat @ Wf.T) + bf
        if Wi is not None:
            gate = gate + (F @ Wi.T)
        mu = sigmoid(gate) * dtp(5.0)
    else:
        mu = dtp(0.0)
    M = active_factor(x, v, act, topology)
    if topology == 1:
        c = torus_christoffel(v, x, R, r) * M + mu * v
    else:
        one = dtp(1.0)
        proj = v @ U
        norm = np.sqrt(np.sum(proj * proj, axis=-1, keepdims=True))
        scale = one / ((one + norm) + dtp(1e-6))
        g = ((proj * proj) * scale) @ W.T
        c = dtp(20.0) * np.tanh((g + mu * v) / dtp(20.0)) * M
    return F - c


_CBRT2 = 2.0 ** (1.0 / 3.0)
_YOSHIDA = ([1 / (2 - _CBRT2) / 2, (1 - 1 / (2 - _CBRT2)) / 2, (1 - 1 / (2 - _CBRT2)) / 2,
             1 / (2 - _CBRT2) / 2],
            [1 / (2 - _CBRT2), -_CBRT2 / (2 - _CBRT2), 1 / (2 - _CBRT2), 1 / (2 - _CBRT2)])
_OMELYAN_XI, _OMELYAN_LAM, _OMELYAN_CHI = 0.1786178958448091, -0.2123418310626054, -0.06626458266981849
_OMELYAN = ([_OMELYAN_XI, _OMELYAN_CHI, 1.0 - 2.0 * (_OMELYAN_CHI + _OMELYAN_XI), _OMELYAN_CHI, _OMELYAN_XI],
            [(1.0 - 2.0 * _OMELYAN_LAM) / 2.0, _OMELYAN_LAM, _OMELYAN_LAM, (1.0 - 2.0 * _OMELYAN_LAM) / 2.0,
             (1.0 - 2.0 * _OMELYAN_LAM) / 2.0])
_DP_A = [[1 / 5], [3 / 40, 9 / 40], [44 / 45, -56 / 15, 32 / 9],
         [19372 / 6561, -25360 / 2187, 64448 / 6561, -212 / 729],
         [9017 / 3168, -355 / 33, 46732 / 5247, 49 / 176, -5103 / 18656]]
_DP_B = [35 / 384, 0, 500 / 1113, 125 / 192, -2187 / 6784, 11 / 84]


def integrator_step(scheme, x, v, F, U, W, Wf, bf, Wi, dt, dt_scale, steps=1, topology=0, R=2.0, r=1.0,
                    act=None):
    """The reference's other integrators (gfn/integrators/runge_kutta/{euler,heun,
    rk4,dormand_prince}.py, gfn/integrators/symplectic/{verlet,yoshida,forest_ruth,
    omelyan}.py), with the combined-form acceleration.  Forest-Ruth and Yoshida
    share their coefficients (theta = 1 / (2 - 2^(1/3)))."""
    dtp = x.dtype.type
    dt = dtp(dt) * dtp(dt_scale)
    wrap = torus_wrap if topology == 1 else (lambda z: z)

    def acc(xx, vv):
        return combined_accel(xx, vv, F, U, W, Wf, bf, Wi, topology, R, r, act)

    for _ in range(steps):
        if scheme == "euler":
            a = acc(x, v)
            x, v = wrap(x + dt * v), v + dt * a
        elif scheme == "heun":
            dv1 = acc(x, v)
            vp = v + dt * dv1
            xp = wrap(x + dt * v)
            dv2 = acc(xp, vp)
            h2 = dt / dtp(2.0)
            x, v = wrap(x + h2 * (v + vp)), v + h2 * (dv1 + dv2)
        elif scheme == "rk4":
            hh = dtp(0.5) * dt
            dv1 = acc(x, v)
            v2, x2 = v + hh * dv1, wrap(x + hh * v)
            dv2 = acc(x2, v2)
            v3, x3 = v + hh * dv2, wrap(x + hh * v2)
            dv3 = acc(x3, v3)
            v4, x4 = v + dt * dv3, wrap(x + dt * v3)
            dv4 = acc(x4, v4)
            s6 = dt / dtp(6.0)
            x = wrap(x + s6 * (v + dtp(2) * v2 + dtp(2) * v3 + v4))
            v = v + s6 * (dv1 + dtp(2) * dv2 + dtp(2) * dv3 + dv4)
        elif scheme == "verlet":
            hh = dtp(0.5) * dt
            vh = v + hh * acc(x, v)
            x = wrap(x + dt * vh)
            v = vh + hh * acc(x, vh)
        elif scheme in ("yoshida", "forest_ruth", "omelyan"):
            cs, ds = _OMELYAN if scheme == "omelyan" else _YOSHIDA
            for c, d in zip(cs, ds):
                x = wrap(x + (dtp(c) * dt) * v)
                v = v + (dtp(d) * dt) * acc(x, v)
        elif scheme in ("rk45", "dormand_prince"):
            kx, kv = [v], [acc(x, v)]
            for row in _DP_A:
                sx = sum((dtp(a) * kx[j] for j, a in enumerate(row)), dtp(0.0))
                sv = sum((dtp(a) * kv[j] for j, a in enumerate(row)), dtp(0.0))
                xs, vs = wrap(x + dt * sx), v + dt * sv
                kx.append(vs)
                kv.append(acc(xs, vs))
            sx = sum((dtp(b) * kx[j] for j, b in enumerate(_DP_B) if b), dtp(0.0))
            sv = sum((dtp(b) * kv[j] for j, b in enumerate(_DP_B) if b), dtp(0.0))
            x, v = wrap(x + dt * sx), v + dt * sv
        else:
            raise ValueError(scheme)
    return x, v


def _gate_mlp(xh, lp, h, topology):
    """RiemannianGating.curvature_net (gfn/layers/gating.py:16-23,38-51)."""
    feat = np.concatenate([np.sin(xh), np.cos(xh)], -1) if topology == 1 else xh
    z = np.tanh((feat @ lp["gW1"][h].T) + lp["gb1"][h])
    return sigmoid(((z @ lp["gW2"][h].T) + lp["gb2"][h]).astype(xh.dtype))


def mlayer_step_generic(x, v, F, lp, heads, base_dt, scheme="leapfrog", topology=0, active=None,
                        context=None):
    """MLayer.forward for the torus and the non-leapfrog integrators
    (gfn/layers/base.py:198-338): per head, the integrator with the stacked
    gates (the leapfrog reads the forget gate only, the others add the input
    gate); mixing reads [sin x, cos x, tanh(v/100)] and wraps x on the torus."""
    B, d = x.shape
    hd = d // heads
    dtp = x.dtype.type
    active = active or {}
    if active.get("recursive_geodesics", {}).get("enabled", False) and context is not None:
        F = F + ((context @ lp["cW"].T) + lp["cb"])          # gfn/layers/base.py:212-214
    sc = softplus(lp["dt_params"].astype(x.dtype))
    dyn = active.get("dynamic_time", {}).get("enabled", False)
    gates = np.ones((heads, B, 1), x.dtype)
    if dyn:
        gates = np.stack([_gate_mlp(x[:, h * hd:(h + 1) * hd], lp, h, topology) for h in range(heads)])
    xo, vo = np.empty_like(x), np.empty_like(v)
    on = active.get("enabled", False)
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        U = lp["U"][h] if "U" in lp else None
        W = lp["W"][h] if "W" in lp else None
        scale = (sc[h] * gates[h]) if dyn else sc[h]
        act = None
        if on:
            rc = active.get("reactive_curvature", {})
            sgc = active.get("singularities", {})
            plast = rc.get("plasticity", 0.1 if topology == 1 else 0.0) if rc.get("enabled", False) else 0.0
            act = dict(plasticity=plast)
            if sgc.get("enabled", False):
                act.update(V=lp["V"][h], Vb=lp["Vb"][h] if topology == 1 else None,
                           thr=sgc.get("threshold", 0.8), strength=sgc.get("strength", 10.0))
        if scheme == "leapfrog":
            xo[:, sl], vo[:, sl] = leapfrog_head_step_gated(x[:, sl], v[:, sl], F[:, sl], U, W, lp["Wf"][h],
                                                            lp["bf"][h], None, base_dt, scale, 1, topology,
                                                            act=act)
        else:
            xo[:, sl], vo[:, sl] = integrator_step(scheme, x[:, sl], v[:, sl], F[:, sl], U, W, lp["Wf"][h],
                                                   lp["bf"][h], lp["Wi"][h], base_dt, scale, 1, topology,
                                                   act=act)
    if heads > 1:
        if topology == 1:
            mix_in = np.concatenate([np.sin(xo), np.cos(xo), np.tanh(vo / dtp(100.0))], -1)
            xn = torus_wrap((mix_in @ lp["Wx"].T) + lp["bx"])
        else:
            xn = rmsnorm((xo @ lp["Wx"].T) + lp["bx"], lp["gx"])
        vn = rmsnorm((vo @ lp["Wv"].T) + lp["bv"], lp["gv"])
    else:
        xn, vn = xo, vo
    return xn, dtp(100.0) * np.tanh(vn / dtp(100.0)), gates[..., 0].T


def manifold_forward_generic(x0, v0, forces, layers, heads, base_dt, scheme="leapfrog", topology=0,
                             active=None):
    """manifold_forward with mlayer_step_generic (gfn/model.py:377-402); the
    per-head gates flow to the next layer as its context (gfn/model.py:385)."""
    B, L, d = forces.shape
    x, v = x0.copy(), v0.copy()
    xs, vs = np.empty((B, L, d), x0.dtype), np.empty((B, L, d), x0.dtype)
    ctx = None
    for t in range(L):
        for lp in layers:
            x, v, ctx = mlayer_step_generic(x, v, forces[:, t], lp, heads, base_dt, scheme, topology,
                                            active, ctx)
        xs[:, t], vs[:, t] = x, v
    return xs, vs, x, v


def rmsnorm(y, g):
    """torch.nn.RMSNorm(d, eps=None): y * rsqrt(mean(y^2) + eps) * g."""
    dt = y.dtype
    ms = np.mean(y * y, axis=-1, keepdims=True)
    return (y * (dt.type(1.0) / np.sqrt(ms + dt.type(_rms_eps(dt))))) * g


def mlayer_step(x, v, F, lp, heads, base_dt):
    """MLayer.forward for the Euclidean leapfrog configuration.

    gfn/layers/base.py:198-338: split heads (:209-217), dt scale =
    softplus(dt_params) (:220,231), per-head integrator (:276-290), concat,
    x' = RMSNorm(out_proj_x(x)), v' = RMSNorm(out_proj_v(v)) (:305-330) when
    heads > 1, then v' = 100 tanh(v'/100) (:335).
    """
    B, d = x.shape
    hd = d // heads
    dtp = x.dtype.type
    scale = softplus(lp["dt_params"].astype(x.dtype))
    xo = np.empty_like(x)
    vo = np.empty_like(v)
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        xh, vh = leapfrog_head_step(x[:, sl], v[:, sl], F[:, sl], lp["U"][h], lp["W"][h],
                                    lp["Wf"][h], lp["bf"][h], base_dt, scale[h])
        xo[:, sl] = xh
        vo[:, sl] = vh
    if heads > 1:
        xn = rmsnorm(xo @ lp["Wx"].T + lp["bx"], lp["gx"])
        vn = rmsnorm(vo @ lp["Wv"].T + lp["bv"], lp["gv"])
    else:
        xn, vn = xo, vo
    vn = dtp(100.0) * np.tanh(vn / dtp(100.0))
    return xn, vn


def manifold_forward(x0, v0, forces, layers, heads, base_dt, mask=None):
    """Manifold.forward loop path without readout.

    gfn/model.py:377-402: for each token t, force = F[:, t] * mask[:, t], then
    every layer in order; x_seq/v_seq collect the state after the last layer.
    x0, v0: [B, d]; forces: [B, L, d].  Returns (x_seq, v_seq, x, v).
    """
    B, L, d = forces.shape
    x, v = x0.copy(), v0.copy()
    xs = np.empty((B, L, d), x0.dtype)
    vs = np.empty((B, L, d), x0.dtype)
    for t in range(L):
        F = forces[:, t]
        if mask is not None:
            F = F * mask[:, t, None].astype(F.dtype)
        for lp in layers:
            x, v = mlayer_step(x, v, F, lp, heads, base_dt)
        xs[:, t] = x
        vs[:, t] = v
    return xs, vs, x, v


def embedding_lookup(ids, table):
    """nn.Embedding forward (gfn/model.py:55, 163)."""
    return table[ids]


def functional_embedding(ids, fp, coord_dim=16, omega_0=30.0):
    """FunctionalEmbedding(mode='binary') forward (gfn/embeddings.py:171-206).

    bits of the id -> {-1, 1} coords -> SIREN (sin(omega_0 * Linear)) x 3 ->
    out_proj -> * impulse_scale -> zero for id 0.  fp holds W0,b0,W1,b1,W2,b2
    (SineLayer linears, gfn/embeddings.py:24-49), Wo, bo, impulse.
    """
    dt = fp["Wo"].dtype
    mask = (1 << np.arange(coord_dim)).astype(np.int64)
    bits = (ids[..., None].astype(np.int64) & mask) > 0
    coords = bits.astype(dt) * dt.type(2) - dt.type(1)
    h = coords
    for i in range(3):
        h = np.sin(dt.type(omega_0) * (h @ fp[f"W{i}"].T + fp[f"b{i}"]))
    out = (h @ fp["Wo"].T + fp["bo"]) * fp["impulse"]
    active = (bits.astype(dt).sum(-1, keepdims=True) > 0).astype(dt)
    return out * active


# ----------------------------------------------------------------------------
# Parallel-scan path
# ----------------------------------------------------------------------------

def scan_sequential(a, x):
    """y_t = a_t y_{t-1} + x_t, y_{-1} = 0 (gfn/scan.py:56-63)."""
    B, L, D = x.shape
    y = np.empty_like(x)
    hcur = np.zeros((B, D), x.dtype)
    for t in range(L):
        hcur = a[:, t] * hcur + x[:, t]
        y[:, t] = hcur
    return y


def parallel_scan(a, x):
    """gfn.scan.parallel_scan: sequential for L < 32, else Hillis-Steele
    doubling with (a2,x2)o(a1,x1) = (a2 a1, a2 x1 + x2) (gfn/scan.py:52-104)."""
    B, L, D = x.shape
    if L < 32:
        return scan_sequential(a, x)
    ca, cx = a.copy(), x.copy()
    steps = int(np.ceil(np.log2(L)))
    for i in range(steps):
        s = 2 ** i
        na = ca.copy()
        nx = cx.copy()
        na[:, s:] = ca[:, s:] * ca[:, :-s]
        nx[:, s:] = ca[:, s:] * cx[:, :-s] + cx[:, s:]
        ca, cx = na, nx
    return cx


def layernorm(x, w, b, eps=1e-5):
    mu = np.mean(x, axis=-1, keepdims=True)
    var = np.mean((x - mu) ** 2, axis=-1, keepdims=True)
    return (x - mu) / np.sqrt(var + x.dtype.type(eps)) * w + b


def parallel_mlayer(force, pp, heads, scan=parallel_scan):
    """ParallelMLayer.forward(None, None, force) (gfn/layers/parallel.py:75-125).

    force = LayerNorm(force); A = sigmoid(to_A(force)); dt = softplus(to_dt(force))
    * 0.1 * 1.5^head; B = to_B(force) * dt; v = scan(A, B); x = scan(1, v * dt).
    pp: ln_w, ln_b, WA, bA, Wdt, bdt, WB, bB.  Returns (x_seq, v_seq).
    """
    dtp = force.dtype.type
    B_, L, D = force.shape
    f = layernorm(force, pp["ln_w"], pp["ln_b"])
    A = sigmoid(f @ pp["WA"].T + pp["bA"])
    scales = np.repeat(np.array([1.5 ** i for i in range(heads)], force.dtype), D // heads)
    dt = softplus(f @ pp["Wdt"].T + pp["bdt"]) * dtp(0.1) * scales
    Bv = (f @ pp["WB"].T + pp["bB"]) * dt
    v_seq = scan(A, Bv)
    x_seq = scan(np.ones_like(v_seq), v_seq * dt)
    return x_seq, v_seq


def manifold_scan_forward(forces, players, heads, scan=parallel_scan):
    """Manifold(use_scan=True) recurrence part (gfn/model.py:171-182): each
    layer's x_seq is the next layer's force.  Returns the last layer's x_seq."""
    cur = forces
    for pp in players:
        cur, _ = parallel_mlayer(cur, pp, heads, scan)
    return cur


# ----------------------------------------------------------------------------
# Backward (BPTT) of the leapfrog loop path
# ----------------------------------------------------------------------------
# The reference's training path is torch autograd through the loop of
# gfn/model.py:377-402 (its fused CUDA backwards are incomplete or excluded for
# leapfrog).  This is the same gradient written out by hand: every layer step
# is recomputed from its stored input state and differentiated in reverse.

def _gamma_fwd(v, U, W):
    dt = v.dtype.type
    p = v @ U
    n = np.sqrt(np.sum(p * p, axis=-1, keepdims=True))
    s = dt(1.0) / ((dt(1.0) + n) + dt(1e-6))
    q = (p * p) * s
    G = dt(20.0) * np.tanh((q @ W.T) / dt(20.0))
    return G, (v, p, n, s, q, G)


def _gamma_bwd(dG, cache, U, W):
    """d/d(v, U, W) of G = 20 tanh(((vU)^2 s) W^T / 20), s = 1/(1+|vU|+1e-6)."""
    v, p, n, s, q, G = cache
    dt = v.dtype.type
    dg = dG * (dt(1.0) - (G / dt(20.0)) ** 2)
    dW = dg.T @ q
    dq = dg @ W
    dp = dq * dt(2.0) * p * s
    ds = np.sum(dq * p * p, axis=-1, keepdims=True)
    dn = -ds * s * s
    safe = np.where(n > 0, n, dt(1.0))
    dp = dp + np.where(n > 0, dn * p / safe, dt(0.0))
    return dp @ U.T, v.T @ dp, dW


def _head_fwd(x, v, F, U, W, Wf, bf, eff, h):
    dt = x.dtype.type
    G1, c1 = _gamma_fwd(v, U, W)
    mu1 = sigmoid(x @ Wf.T + bf) * dt(5.0)
    D1 = dt(1.0) + h * mu1
    vh = (v + h * (F - G1)) / D1
    x2 = x + eff * vh
    G2, c2 = _gamma_fwd(vh, U, W)
    mu2 = sigmoid(x2 @ Wf.T + bf) * dt(5.0)
    D2 = dt(1.0) + h * mu2
    v2 = (vh + h * (F - G2)) / D2
    return x2, v2, (x, v, F, G1, c1, mu1, D1, vh, x2, G2, c2, mu2, D2, v2)


def _head_bwd(dx2, dv2, cache, U, W, Wf, eff, h):
    x, v, F, G1, c1, mu1, D1, vh, x2, G2, c2, mu2, D2, v2 = cache
    dt = x.dtype.type
    dN2 = dv2 / D2
    dD2 = -dv2 * v2 / D2
    dmu2 = dD2 * h
    dh = np.sum(dD2 * mu2)
    dvh = dN2.copy()
    dF = dN2 * h
    dG2 = -dN2 * h
    dh += np.sum(dN2 * (F - G2))
    dz2 = dmu2 * mu2 * (dt(1.0) - mu2 / dt(5.0))
    dx2t = dx2 + dz2 @ Wf
    dWf = dz2.T @ x2
    dbf = dz2.sum(0)
    dvg, dU, dW = _gamma_bwd(dG2, c2, U, W)
    dvh += dvg
    dx = dx2t.copy()
    dvh += eff * dx2t
    deff = np.sum(dx2t * vh)
    dN1 = dvh / D1
    dD1 = -dvh * vh / D1
    dmu1 = dD1 * h
    dh += np.sum(dD1 * mu1)
    dv = dN1.copy()
    dF += dN1 * h
    dG1 = -dN1 * h
    dh += np.sum(dN1 * (F - G1))
    dz1 = dmu1 * mu1 * (dt(1.0) - mu1 / dt(5.0))
    dx += dz1 @ Wf
    dWf += dz1.T @ x
    dbf += dz1.sum(0)
    dvg, dU1, dW1 = _gamma_bwd(dG1, c1, U, W)
    dv += dvg
    dU += dU1
    dW += dW1
    deff += dt(0.5) * dh
    return dx, dv, dF, dict(U=dU, W=dW, Wf=dWf, bf=dbf, eff=deff)


def _rms_fwd(z, g):
    dt = z.dtype
    ms = np.mean(z * z, axis=-1, keepdims=True)
    r = dt.type(1.0) / np.sqrt(ms + dt.type(_rms_eps(dt)))
    y = z * r
    return y * g, (z, r, y)


def _rms_bwd(dout, cache, g):
    z, r, y = cache
    d = z.shape[-1]
    dy = dout * g
    dg = np.sum(dout * y, axis=0)
    dz = r * dy - (r ** 3 / z.dtype.type(d)) * z * np.sum(dy * z, axis=-1, keepdims=True)
    return dz, dg


def mlayer_step_cached(x, v, F, lp, heads, base_dt):
    """mlayer_step that also returns what its backward needs."""
    B, d = x.shape
    hd = d // heads
    dtp = x.dtype.type
    sc = softplus(lp["dt_params"].astype(x.dtype))
    xo = np.empty_like(x)
    vo = np.empty_like(v)
    hc = []
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        eff = dtp(base_dt) * sc[h]
        hh = dtp(0.5) * eff
        xh, vh, c = _head_fwd(x[:, sl], v[:, sl], F[:, sl], lp["U"][h], lp["W"][h], lp["Wf"][h],
                              lp["bf"][h], eff, hh)
        xo[:, sl] = xh
        vo[:, sl] = vh
        hc.append((c, eff, hh))
    if heads > 1:
        zx = xo @ lp["Wx"].T + lp["bx"]
        zv = vo @ lp["Wv"].T + lp["bv"]
        xn, cx = _rms_fwd(zx, lp["gx"])
        w, cv = _rms_fwd(zv, lp["gv"])
        mix = (xo, vo, cx, cv)
    else:
        xn, w, mix = xo, vo, None
    vn = dtp(100.0) * np.tanh(w / dtp(100.0))
    return xn, vn, (hc, mix, vn, sc)


def mlayer_step_backward(dxn, dvn, cache, lp, heads, base_dt):
    """Gradients of one MLayer step: (dx_in, dv_in, dF, param grads)."""
    hc, mix, vn, sc = cache
    dtp = dxn.dtype.type
    B, d = dxn.shape
    hd = d // heads
    grads = {}
    dw = dvn * (dtp(1.0) - (vn / dtp(100.0)) ** 2)
    if heads > 1:
        xo, vo, cx, cv = mix
        dzx, grads["gx"] = _rms_bwd(dxn, cx, lp["gx"])
        dzv, grads["gv"] = _rms_bwd(dw, cv, lp["gv"])
        grads["bx"] = dzx.sum(0)
        grads["bv"] = dzv.sum(0)
        grads["Wx"] = dzx.T @ xo
        grads["Wv"] = dzv.T @ vo
        dxo = dzx @ lp["Wx"]
        dvo = dzv @ lp["Wv"]
    else:
        dxo, dvo = dxn, dw
    dx = np.empty_like(dxn)
    dv = np.empty_like(dxn)
    dF = np.empty_like(dxn)
    gU = np.empty_like(lp["U"])
    gW = np.empty_like(lp["W"])
    gWf = np.empty_like(lp["Wf"])
    gbf = np.empty_like(lp["bf"])
    gdt = np.empty_like(lp["dt_params"])
    th = lp["dt_params"].astype(dxn.dtype)
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        c, eff, hh = hc[h]
        a, b, f, g = _head_bwd(dxo[:, sl], dvo[:, sl], c, lp["U"][h], lp["W"][h], lp["Wf"][h],
                               eff, hh)
        dx[:, sl], dv[:, sl], dF[:, sl] = a, b, f
        gU[h], gW[h], gWf[h], gbf[h] = g["U"], g["W"], g["Wf"], g["bf"]
        # eff = base_dt * softplus(theta): d theta = d eff * base_dt * sigmoid(theta)
        gdt[h] = g["eff"] * dtp(base_dt) * sigmoid(th[h:h + 1])[0]
    grads.update(U=gU, W=gW, Wf=gWf, bf=gbf, dt_params=gdt)
    return dx, dv, dF, grads


def manifold_backward(x0, v0, forces, layers, heads, base_dt, gx_seq, gv_seq,
                      gx_final=None, gv_final=None, mask=None):
    """Gradients of L = <gx_seq, x_seq> + <gv_seq, v_seq> (+ <gx_final, x_L> +
    <gv_final, v_L>) through manifold_forward.  Returns dict with x0, v0
    ([B, d]), forces ([B, L, d]) and 'layers' (list of per-layer param grads)."""
    B, L, d = forces.shape
    NL = len(layers)
    x, v = x0.copy(), v0.copy()
    inputs = []
    for t in range(L):
        F = forces[:, t] if mask is None else forces[:, t] * mask[:, t, None].astype(forces.dtype)
        for lp in layers:
            inputs.append((x, v, F))
            x, v = mlayer_step(x, v, F, lp, heads, base_dt)
    dx = np.zeros_like(x0) if gx_final is None else gx_final.astype(x0.dtype).copy()
    dv = np.zeros_like(v0) if gv_final is None else gv_final.astype(v0.dtype).copy()
    dforces = np.zeros_like(forces)
    lg = [None] * NL
    for t in reversed(range(L)):
        dx = dx + gx_seq[:, t]
        dv = dv + gv_seq[:, t]
        dF_t = np.zeros_like(x0)
        for l in reversed(range(NL)):
            xi, vi, F = inputs[t * NL + l]
            _, _, cache = mlayer_step_cached(xi, vi, F, layers[l], heads, base_dt)
            dx, dv, dF, g = mlayer_step_backward(dx, dv, cache, layers[l], heads, base_dt)
            dF_t += dF
            lg[l] = g if lg[l] is None else {k: lg[l][k] + g[k] for k in g}
        dforces[:, t] = dF_t if mask is None else dF_t * mask[:, t, None].astype(forces.dtype)
    return dict(x0=dx, v0=dv, forces=dforces, layers=lg)
