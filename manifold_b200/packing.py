"""Gathers MLayer parameters into the stacked form the C ABI takes and
caches the packed device buffer until a parameter changes.

The stacks are the ones the reference assembles for its fused launcher
(gfn/model.py:222-293: U/W/forget-gate stacks over layers x heads) plus
every layer's mixing weights (the reference passes only layer 0's,
gfn/model.py:299-302; the leapfrog loop it actually runs uses each layer's
own, gfn/layers/base.py:313-330).
"""
import torch

from .cuda import ops


def layer_tensors(layers):
    """Parameter tensors of `layers` in pack order."""
    U, W, Wf, bf, dtp, mix = [], [], [], [], [], []
    for layer in layers:
        for ch in layer.christoffels:
            U.append(ch.U)
            W.append(ch.W)
            Wf.append(ch.forget_gate.weight)
            bf.append(ch.forget_gate.bias)
        dtp.append(layer.dt_params)
        if layer.heads > 1:
            mix.append((layer.out_proj_x.weight, layer.out_proj_x.bias, layer.mixed_norm_x.weight,
                        layer.out_proj_v.weight, layer.out_proj_v.bias, layer.mixed_norm_v.weight))
    return U, W, Wf, bf, dtp, mix


def _key(tensors):
    return tuple((t.data_ptr(), t._version, tuple(t.shape)) for t in tensors)


def stacks(layers):
    U, W, Wf, bf, dtp, mix = layer_tensors(layers)
    out = dict(U=torch.stack(U), W=torch.stack(W), Wf=torch.stack(Wf), bf=torch.stack(bf),
               dtp=torch.cat(dtp))
    if mix:
        names = ("Wx", "bx", "gx", "Wv", "bv", "gv")
        for i, n in enumerate(names):
            out[n] = torch.stack([m[i] for m in mix])
    return out


class PackCache:
    """Holds the packed weights of a list of layers; re-packs on change.

    `layered=True` gives the layout of the layer-by-layer (large batch)
    path; both layouts are cached independently.
    """

    def __init__(self):
        self._key = None
        self.packed = None
        self.meta = None
        self._lay = None

    def get(self, layers, layered=False):
        U, W, Wf, bf, dtp, mix = layer_tensors(layers)
        flat = U + W + Wf + bf + dtp + [t for m in mix for t in m]
        key = _key(flat)
        if layered:
            if self._lay is None or self._lay[0] != key:
                with torch.no_grad():
                    s = stacks(layers)
                    mixt = (s["Wx"], s["bx"], s["gx"], s["Wv"], s["bv"], s["gv"])
                    packed, meta = ops.leapfrog_layered_pack(s["U"], s["W"], s["Wf"], s["bf"],
                                                             s["dtp"], mixt)
                self._lay = (key, packed, meta)
            return self._lay[1], self._lay[2]
        if key != self._key:
            with torch.no_grad():
                s = stacks(layers)
                mixt = None
                if "Wx" in s:
                    mixt = (s["Wx"], s["bx"], s["gx"], s["Wv"], s["bv"], s["gv"])
                self.packed, self.meta = ops.leapfrog_pack(s["U"], s["W"], s["Wf"], s["bf"],
                                                           s["dtp"], mixt)
                if mixt is None:
                    # heads == 1: layers are stacked on the head axis
                    self.meta = dict(self.meta, num_layers=len(layers))
            self._key = key
        return self.packed, self.meta
