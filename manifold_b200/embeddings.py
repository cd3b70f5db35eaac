"""Token -> force embeddings (mirror of gfn/embeddings.py).

FunctionalEmbedding (the one the LM-shaped configuration uses) runs as one
fused SIREN kernel over all [B, L] tokens; ImplicitEmbedding keeps the
reference's module and evaluates with torch GPU ops (it is not on any
benchmarked path).
"""
import numpy as np
import torch
import torch.nn as nn

from ._lib import GfnError, require_cuda
from .cuda import ops


class SineLayer(nn.Module):
    """sin(omega_0 * Linear(x)) with SIREN init (gfn/embeddings.py:24-49)."""

    def __init__(self, in_features, out_features, bias=True, is_first=False, omega_0=30.0):
        super().__init__()
        self.omega_0 = omega_0
        self.is_first = is_first
        self.linear = nn.Linear(in_features, out_features, bias=bias)
        self.init_weights()

    def init_weights(self):
        with torch.no_grad():
            if self.is_first:
                bound = 1 / self.linear.weight.size(1)
            else:
                bound = np.sqrt(6 / self.linear.weight.size(1)) / self.omega_0
            self.linear.weight.uniform_(-bound, bound)

    def forward(self, x):
        return torch.sin(self.omega_0 * self.linear(x))


class ImplicitEmbedding(nn.Module):
    """Coordinate table -> SIREN -> Linear, x1.5 (gfn/embeddings.py:52-119)."""

    def __init__(self, vocab_size, emb_dim, coord_dim=16, hidden_dim=64, layers=2):
        super().__init__()
        self.vocab_size = vocab_size
        self.emb_dim = emb_dim
        self.coord_dim = coord_dim
        self.coords = nn.Embedding(vocab_size, coord_dim)
        nn.init.uniform_(self.coords.weight, -1.0, 1.0)
        net = [SineLayer(coord_dim, hidden_dim, is_first=True, omega_0=30.0)]
        for _ in range(layers):
            net.append(SineLayer(hidden_dim, hidden_dim, is_first=False, omega_0=30.0))
        self.net = nn.Sequential(*net)
        self.out_proj = nn.Linear(hidden_dim, emb_dim)
        with torch.no_grad():
            nn.init.xavier_uniform_(self.out_proj.weight)
            nn.init.zeros_(self.out_proj.bias)

    def forward(self, input_ids):
        require_cuda(input_ids)
        return self.out_proj(self.net(self.coords(input_ids))) * 1.5


class FunctionalEmbedding(nn.Module):
    """Zero-lookup embedding: id -> bits -> SIREN -> force
    (gfn/embeddings.py:121-206).  Mode 'binary' runs on the fused kernel."""

    def __init__(self, vocab_size, emb_dim, coord_dim=16, hidden_dim=64, layers=2, mode="binary",
                 impulse_scale=1.0, omega_0=30.0):
        super().__init__()
        self.mode = mode
        self.coord_dim = coord_dim
        self.omega_0 = omega_0
        self.impulse_scale = nn.Parameter(torch.tensor(impulse_scale), requires_grad=True)
        if self.mode == "linear":
            self.net = nn.Identity()
            self.out_proj = nn.Linear(self.coord_dim, emb_dim)
            with torch.no_grad():
                nn.init.constant_(self.out_proj.weight, 1.0)
                nn.init.zeros_(self.out_proj.bias)
        else:
            net = [SineLayer(self.coord_dim, hidden_dim, is_first=True, omega_0=self.omega_0)]
            for _ in range(layers):
                net.append(SineLayer(hidden_dim, hidden_dim, is_first=False, omega_0=self.omega_0))
            self.net = nn.Sequential(*net)
            self.out_proj = nn.Linear(hidden_dim, emb_dim)
            with torch.no_grad():
                self.out_proj.weight.data *= 1.5
                nn.init.zeros_(self.out_proj.bias)
        if self.mode == "sinusoidal":
            if coord_dim % 2 != 0:
                self.coord_dim += 1
            freqs = torch.exp(torch.arange(0, self.coord_dim, 2).float()
                              * -(np.log(10000.0) / self.coord_dim))
            self.register_buffer("freqs", freqs)
        self.hidden_dim = hidden_dim
        self.n_layers = layers
        self.out_dtype = torch.float32

    def _fused_ok(self):
        return (self.mode == "binary" and self.coord_dim == 16 and self.hidden_dim == 64
                and self.n_layers == 2)

    def forward(self, input_ids, out_dtype=None):
        require_cuda(input_ids)
        if not self._fused_ok():
            raise GfnError(f"FunctionalEmbedding mode={self.mode!r} coord_dim={self.coord_dim} "
                           "is not implemented on this build (binary/16/64/2 is)")
        n = self.net
        return ops.functional_embedding(
            input_ids, n[0].linear.weight, n[0].linear.bias, n[1].linear.weight, n[1].linear.bias,
            n[2].linear.weight, n[2].linear.bias, self.out_proj.weight, self.out_proj.bias,
            self.impulse_scale, self.omega_0, out_dtype=out_dtype or self.out_dtype)
