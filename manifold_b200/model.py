"""Manifold sequence model (mirror of gfn/model.py) on the B200 kernels.

Same constructor, parameters, initialisation order and forward signature as
the reference.  The leapfrog loop path (gfn/model.py:377-402: for every
token, every layer) runs as ONE persistent kernel launch for the whole
[B, L] sequence; the token embedding gather is fused into it.  The scan
path (use_scan=True, gfn/model.py:171-188) runs ParallelMLayer per layer.
The readout (LayerNorm + Linear) is applied to the whole x_seq afterwards
with torch (cuBLAS); it is not part of the recurrence.
"""
import torch
import torch.nn as nn

from ._lib import GfnError, require_cuda
from .cuda import ops
from .embeddings import FunctionalEmbedding, ImplicitEmbedding
from .layers import LAYERED_MIN_ELEMS, MLayer, ParallelMLayer, use_layered_path  # noqa: F401
from .packing import PackCache


class ImplicitReadout(nn.Module):
    """MLP readout to coordinate logits (gfn/readout.py:4-72)."""

    def __init__(self, dim, coord_dim, temp_init=1.0, temp_final=0.2, topology=0):
        super().__init__()
        self.topology = topology
        self.is_torus = topology == 1
        in_dim = dim * 2 if self.is_torus else dim
        self.mlp = nn.Sequential(nn.Linear(in_dim, dim), nn.GELU(), nn.Linear(dim, coord_dim))
        for module in self.mlp.modules():
            if isinstance(module, nn.Linear):
                module.is_readout = True
        self.temp_init = temp_init
        self.temp_final = temp_final
        self.register_buffer("training_step", torch.tensor(0))
        self.register_buffer("max_steps", torch.tensor(1000))

    def forward(self, x):
        x_emb = torch.cat([torch.sin(x), torch.cos(x)], dim=-1) if self.is_torus else x
        return self.mlp(x_emb) * 10.0

    def update_step(self):
        if self.training:
            self.training_step += 1

    def set_max_steps(self, max_steps):
        self.max_steps = torch.tensor(max_steps)


class Manifold(nn.Module):
    """Sequence model evolving (x, v) by leapfrog geodesic flow.

    forward(input_ids, attention_mask, state, force_manual, collect_christ)
    returns (logits, (x, v), christoffels, v_seq, x_seq, all_forces) like
    gfn/model.py:142-402 (v_seq/x_seq as lists of [B, d] per token).
    """

    def __init__(self, vocab_size, dim=256, depth=4, rank=32, heads=4, integrator_type="heun",
                 base_dt=1.0, use_scan=False, physics_config=None, impulse_scale=None,
                 holographic=False):
        super().__init__()
        self.dim = dim
        self.depth = depth
        self.heads = heads
        self.integrator_type = integrator_type
        self.use_scan = use_scan
        self.physics_config = physics_config or {}
        self.holographic = holographic or self.physics_config.get("holographic", False)
        emb_cfg = self.physics_config.get("embedding", {})
        emb_type = emb_cfg.get("type", "standard")
        if emb_type == "implicit":
            self.embedding = ImplicitEmbedding(vocab_size, dim, coord_dim=emb_cfg.get("coord_dim", 16))
        elif emb_type == "functional":
            imp = impulse_scale if impulse_scale is not None else emb_cfg.get("impulse_scale", 1.0)
            self.embedding = FunctionalEmbedding(vocab_size, dim, coord_dim=emb_cfg.get("coord_dim", 16),
                                                 mode=emb_cfg.get("mode", "binary"), impulse_scale=imp,
                                                 omega_0=emb_cfg.get("omega_0", 30.0))
        else:
            self.embedding = nn.Embedding(vocab_size, dim)
        if self.physics_config.get("fractal", {}).get("enabled", False):
            raise GfnError("fractal layers are not implemented on this build")
        self.layers = nn.ModuleList()
        for idx in range(depth):
            if use_scan:
                self.layers.append(ParallelMLayer(dim, heads=heads, physics_config=self.physics_config))
            else:
                self.layers.append(MLayer(dim, heads=heads, rank=rank, base_dt=base_dt,
                                          integrator_type=integrator_type,
                                          physics_config=self.physics_config, layer_idx=idx,
                                          total_depth=depth))
        readout_type = self.physics_config.get("readout", {}).get("type", "standard")
        self.readout_norm = nn.LayerNorm(dim)
        self.readout_split = True  # False: plain fp32 torch matmul for the readout
        if readout_type in ("implicit", "binary"):
            coord_dim = emb_cfg.get("coord_dim", 16)
            self.readout = nn.Identity() if self.holographic else ImplicitReadout(dim, coord_dim)
        else:
            self.readout = nn.Linear(dim, vocab_size)
        self.x0 = nn.Parameter(torch.randn(1, dim) * 0.02)
        self.v0 = nn.Parameter(torch.randn(1, dim) * 0.01)
        self.apply(self._init_weights)
        self.return_forces = True
        self.force_dtype = torch.float32
        self._pack = PackCache()

    def _init_weights(self, module):
        # Same rule and traversal as gfn/model.py:119-140.
        if isinstance(module, FunctionalEmbedding):
            return
        if hasattr(self, "embedding") and isinstance(self.embedding, FunctionalEmbedding):
            emb_params = set(self.embedding.parameters())
            mod_params = set(module.parameters())
            if mod_params.issubset(emb_params) and len(mod_params) > 0:
                return
        if isinstance(module, nn.Linear):
            std = 0.1 if hasattr(module, "is_readout") else 0.02
            nn.init.normal_(module.weight, mean=0.0, std=std)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
        elif isinstance(module, nn.LayerNorm):
            nn.init.zeros_(module.bias)
            nn.init.ones_(module.weight)

    # ------------------------------------------------------------------
    def _forces(self, input_ids, force_manual):
        if force_manual is not None:
            return force_manual
        if isinstance(self.embedding, FunctionalEmbedding):
            return self.embedding(input_ids, out_dtype=self.force_dtype)
        return self.embedding(input_ids)

    def _apply_readout(self, out):
        """The readout: nn.Linear through the split-fp16 tensor-core GEMMs
        (~1e-6 relative error, manifold_b200.readout), other readouts as they are."""
        if isinstance(self.readout, nn.Linear) and out.is_cuda and self.readout_split:
            from .readout import readout_linear
            return readout_linear(out, self.readout)
        return self.readout(out)

    def _use_layered(self, batch):
        """Layer-by-layer path (head-step kernel + fp32 GEMM mixing) for
        large batches, the fused persistent kernel otherwise.  `recurrence_path`
        ("auto", "fused", "layered") overrides the choice."""
        return use_layered_path(getattr(self, "recurrence_path", "auto"), self.heads, self.dim, batch)

    def recurrence(self, input_ids=None, attention_mask=None, state=None, force_manual=None,
                   want_v_seq=True):
        """The recurrence alone: (x_seq [B,L,d], v_seq [B,L,d] or None, (x, v), forces).

        `forces` is None when the embedding gather was fused into the kernel.
        """
        if self.use_scan:
            raise GfnError("recurrence() is the leapfrog loop path; use forward() for use_scan")
        src = force_manual if force_manual is not None else input_ids
        require_cuda(src)
        B = src.shape[0]
        if self.layers[0].generic:
            return self._generic_recurrence(input_ids, attention_mask, state, force_manual, want_v_seq)
        layered = self._use_layered(B)
        packed, meta = self._pack.get(list(self.layers), layered=layered)
        seq = ops.leapfrog_layered_sequence if layered else ops.leapfrog_sequence
        if state is None:
            x, v = self.x0, self.v0
        else:
            x, v = state
        mask = attention_mask
        base_dt = self.layers[0].base_dt
        if force_manual is None and isinstance(self.embedding, nn.Embedding):
            x_seq, v_seq, xf, vf = seq(x, v, packed, meta, base_dt, ids=input_ids,
                                       table=self.embedding.weight, mask=mask, want_v_seq=want_v_seq)
            forces = None
        else:
            forces = self._forces(input_ids, force_manual)
            x_seq, v_seq, xf, vf = seq(x, v, packed, meta, base_dt, forces=forces, mask=mask,
                                       want_v_seq=want_v_seq)
        return x_seq, v_seq, (xf, vf), forces

    def _generic_recurrence(self, input_ids, attention_mask, state, force_manual, want_v_seq):
        """Token-by-token loop of gfn/model.py:377-402 for the torus and the
        non-leapfrog integrators (one multi-scheme integrator launch plus the
        head mixing per layer and token)."""
        forces = self._forces(input_ids, force_manual)
        B, L = forces.shape[:2]
        if state is None:
            x = self.x0.expand(B, -1)
            v = self.v0.expand(B, -1)
        else:
            x, v = state
        xs, vs = [], []
        context = None
        for t in range(L):
            f = forces[:, t].to(torch.float32)
            if attention_mask is not None:
                f = f * attention_mask[:, t].unsqueeze(-1).float()
            for layer in self.layers:
                x, v, context, _ = layer(x, v, f, context)
            xs.append(x)
            vs.append(v)
        x_seq = torch.stack(xs, 1)
        v_seq = torch.stack(vs, 1) if want_v_seq else None
        return x_seq, v_seq, (x, v), forces

    def forward(self, input_ids=None, attention_mask=None, state=None, force_manual=None,
                collect_christ=False):
        if collect_christ:
            raise GfnError("collect_christ is not supported by the fused kernels")
        if self.use_scan:
            forces = self._forces(input_ids, force_manual)
            require_cuda(forces)
            cur = forces
            for layer in self.layers:
                cur, _, _, _ = layer(None, None, force=cur)
            x_final = cur if self.holographic else self.readout_norm(cur)
            logits = self.readout(x_final)
            return logits, (x_final[:, -1], None), []
        train = torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters())
        if train and not self.layers[0].training_generic():
            from .training import manifold_train_forward
            return manifold_train_forward(self, input_ids, attention_mask, state, force_manual)
        if train and self.training and not self.layers[0].generic:
            # head dims beyond the fused BPTT kernels: the generic (layer by
            # layer, per-head autograd) path
            x_seq, v_seq, (x, v), forces = self._generic_recurrence(input_ids, attention_mask, state,
                                                                    force_manual, True)
        else:
            x_seq, v_seq, (x, v), forces = self.recurrence(input_ids, attention_mask, state, force_manual)
        if forces is None and self.return_forces:
            forces = self.embedding(input_ids)
        out = x_seq if self.holographic else self.readout_norm(x_seq)
        logits = self._apply_readout(out)
        return logits, (x, v), [], list(v_seq.unbind(1)), list(x_seq.unbind(1)), forces

    @torch.no_grad()
    def generate(self, prompt_ids, max_new_tokens=50, temperature=1.0, top_k=None, top_p=None):
        """Autoregressive sampling with O(1) streamed state (gfn/model.py:404-469;
        the reference unpacks 3 values from its 6-tuple there and fails)."""
        self.eval()
        logits, state = self(prompt_ids)[:2]
        generated = prompt_ids.tolist()[0]

        def sample_next(lg):
            nl = lg[:, -1, :] / temperature
            if top_k is not None:
                vals, _ = torch.topk(nl, top_k)
                nl[nl < vals[:, [-1]]] = -float("Inf")
            if top_p is not None:
                sl, si = torch.sort(nl, descending=True)
                cp = torch.cumsum(torch.softmax(sl, dim=-1), dim=-1)
                rm = cp > top_p
                rm[..., 1:] = rm[..., :-1].clone()
                rm[..., 0] = 0
                nl[rm.scatter(1, si, rm)] = -float("Inf")
            if top_k is None and top_p is None:
                return torch.argmax(nl, dim=-1, keepdim=True)
            return torch.multinomial(torch.softmax(nl, dim=-1), num_samples=1)

        tok = sample_next(logits)
        generated.append(tok.item())
        for _ in range(max_new_tokens - 1):
            logits, state = self(tok, state=state)[:2]
            tok = sample_next(logits)
            generated.append(tok.item())
        return generated
