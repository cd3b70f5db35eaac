"""The allocation-free scan entry point, checked against the workspace one.

gfn_parallel_scan_noalloc serves callers that cannot allocate device memory
where they run the scan (allocator callbacks, plugins whose host owns all
allocations, fixed memory budgets): its scratch is a fixed array inside the
library.  This file is collected last so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from manifold_b200 import _lib
from tests.parity import rowwise_close

pytestmark = pytest.mark.gpu


def _scan_noalloc(a, x):
    y = torch.empty_like(x)
    B, L, D = x.shape
    _lib.call("gfn_parallel_scan_noalloc", _lib.ptr(a), _lib.ptr(x), _lib.ptr(y), B, L, D,
              _lib.stream_of(x.device))
    return y


def _scan_workspace(a, x):
    y = torch.empty_like(x)
    B, L, D = x.shape
    n = _lib.load().gfn_parallel_scan_workspace_floats(B, L, D)
    ws = torch.empty(int(n), device=x.device, dtype=torch.float32)
    _lib.call("gfn_parallel_scan", _lib.ptr(a), _lib.ptr(x), _lib.ptr(y), _lib.ptr(ws), ws.numel(),
              B, L, D, _lib.stream_of(x.device))
    return y


def test_noalloc_scan_matches_workspace_scan_twice():
    rng = np.random.default_rng(42)
    # small batch x dim with a long time axis: the time-split path that uses
    # the static scratch; the second call has other sizes and data so stale
    # contents of the shared array would show.
    for B, L, D in ((2, 4096, 8), (3, 2500, 16)):
        a = torch.as_tensor(rng.uniform(0.8, 1.0, (B, L, D)).astype(np.float32)).cuda()
        x = torch.as_tensor(rng.standard_normal((B, L, D)).astype(np.float32)).cuda()
        y0 = _scan_workspace(a, x)
        y1 = _scan_noalloc(a, x)
        torch.cuda.synchronize()
        rowwise_close(y1.cpu().numpy(), y0.cpu().numpy(), 1e-5, 1e-5, f"noalloc {B}x{L}x{D}")
        y2 = _scan_noalloc(None, x)  # a == 1: running sum
        rowwise_close(y2.cpu().numpy(), np.cumsum(x.cpu().numpy().astype(np.float64), 1),
                      1e-5, 1e-4, "noalloc cumsum")


def test_noalloc_scan_rejects_sizes_beyond_its_scratch():
    x = torch.zeros(1, 1, 4, device="cuda")
    lib = _lib.load()
    st = lib.gfn_parallel_scan_noalloc(None, x.data_ptr(), x.data_ptr(), 1024, 1, 1024,
                                       _lib.stream_of(x.device))
    assert st == 1
    assert b"static scratch limit" in lib.gfn_last_error_message()
