"""The readout nn.Linear(d -> vocab) (gfn/model.py:393-397) on the tensor
cores with ~22-bit products (~1e-6 relative error, a few float32 ulps).

The reference computes logits = out W^T + b and, in training, the two
backward products dout = dlogits W and dW = dlogits^T out, all in fp32.
Here each product runs as one fp16 tensor-core GEMM over operands split into
two fp16 pieces (gfn_split_f16 / gfn_gemm_split_f16 in the C ABI: K' = 3K,
dropped terms below 2^-22 of each product, per-matrix power-of-two scaling so
any magnitude fits).  Rows are processed in chunks so the split operands stay
a few GB.
"""
import torch

from . import _lib
from ._lib import call, ptr

# rows per chunk: the split logit gradient of a chunk is 6 * rows * vocab bytes
CHUNK_ROWS = 16384


def _split(x, k_along_rows, role_b):
    """fp16 pieces of fp32 matrix x [rows, cols] along K; returns (pieces, scale slot)."""
    rows, cols = x.shape
    shape = (3 * rows, cols) if k_along_rows else (rows, 3 * cols)
    out = torch.empty(shape, device=x.device, dtype=torch.float16)
    sc = torch.empty(2, device=x.device, dtype=torch.float32)
    call("gfn_split_f16", ptr(x), rows, cols, 1 if k_along_rows else 0, 1 if role_b else 0, ptr(out),
         ptr(sc), _lib.stream_of(x.device))
    return out, sc


def _gemm(M, N, K, a2, sa, a_k_rows, b2, sb, b_k_rows, c, beta=0.0):
    ab = torch.empty(3, device=c.device, dtype=torch.float32)
    call("gfn_gemm_split_f16", M, N, K, ptr(a2), 1 if a_k_rows else 0, ptr(b2), 1 if b_k_rows else 0,
         ptr(sa), ptr(sb), float(beta), ptr(c), ptr(ab), _lib.stream_of(c.device))
    return c


class SplitLinear(torch.autograd.Function):
    """y [M, d], W [V, d], b [V] -> y W^T + b, fp32 in and out."""

    @staticmethod
    def forward(ctx, y, W, b):
        y = y.detach().contiguous().float()
        W = W.detach().contiguous().float()
        M, d = y.shape
        V = W.shape[0]
        out = torch.empty(M, V, device=y.device, dtype=torch.float32)
        w2, sw = _split(W, False, True)  # B' = W^T: K = d along W's columns
        tc = d <= 512 and d % 32 == 0 and V % 64 == 0
        bias = b.detach().float().contiguous() if b is not None else None
        alpha = torch.empty(4, device=y.device, dtype=torch.float32)
        for r0 in range(0, M, CHUNK_ROWS):
            yc = y[r0:r0 + CHUNK_ROWS]
            y2, sy = _split(yc, False, False)
            if tc:  # the library's tcgen05 GEMM, bias added in its epilogue
                call("gfn_gemm_split_f16_tc", yc.shape[0], V, d, ptr(y2), ptr(w2), ptr(sy), ptr(sw), ptr(bias),
                     ptr(out[r0:r0 + CHUNK_ROWS]), ptr(alpha), _lib.stream_of(y.device))
            else:
                _gemm(yc.shape[0], V, d, y2, sy, False, w2, sw, False, out[r0:r0 + CHUNK_ROWS])
        if b is not None and not tc:
            out += bias
        ctx.save_for_backward(y, W)
        ctx.has_bias = b is not None
        return out

    @staticmethod
    def backward(ctx, g):
        y, W = ctx.saved_tensors
        g = g.contiguous().float()
        M, d = y.shape
        V = W.shape[0]
        dy = torch.empty_like(y) if ctx.needs_input_grad[0] else None
        dW = torch.zeros_like(W) if ctx.needs_input_grad[1] else None
        wr = _split(W, True, True) if dy is not None else None  # B' = W: K = V along W's rows
        for r0 in range(0, M, CHUNK_ROWS):
            gc = g[r0:r0 + CHUNK_ROWS]
            m = gc.shape[0]
            if dy is not None:
                g2, sg = _split(gc, False, False)  # A' = g: K = V along columns
                _gemm(m, d, V, g2, sg, False, wr[0], wr[1], True, dy[r0:r0 + CHUNK_ROWS])
                del g2
            if dW is not None:
                gt, sgt = _split(gc, True, False)  # A' = g^T: K = rows
                yt, syt = _split(y[r0:r0 + CHUNK_ROWS], True, True)  # B' = y: K = rows
                _gemm(V, d, m, gt, sgt, True, yt, syt, True, dW, beta=0.0 if r0 == 0 else 1.0)
                del gt, yt
        db = g.sum(0) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dy, dW, db


def readout_linear(out, linear):
    """linear(out) for out [..., d] through the split-fp16 tensor-core GEMMs."""
    shp = out.shape
    y = out.reshape(-1, shp[-1])
    logits = SplitLinear.apply(y, linear.weight, linear.bias)
    return logits.reshape(*shp[:-1], linear.weight.shape[0])
