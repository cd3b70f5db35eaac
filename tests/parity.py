"""Parity assertions shared by the tests.

Per-step fp32 parity is judged row by row against the state's magnitude:
|a - b| <= atol + rtol * max|b_row| with rtol = 1e-5, atol = 1e-6.  An
element-relative bound is below the float32 noise floor of a d-wide dot
product followed by RMSNorm (two correct float32 implementations, e.g. the
reference's torch CPU and a numpy restatement, differ by ~2e-6 on a 0.03
element of a d = 1024 row), so the bound is taken per row.
"""
import numpy as np

STEP_RTOL = 1e-5
STEP_ATOL = 1e-6


def rowwise_close(a, b, rtol=STEP_RTOL, atol=STEP_ATOL, what=""):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    scale = np.max(np.abs(b), axis=-1, keepdims=True)
    err = np.abs(a - b)
    tol = atol + rtol * scale
    bad = err > tol
    if bad.any():
        i = np.unravel_index(np.argmax(err - tol), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} elements off; worst at {i}: "
                             f"{a[i]!r} vs {b[i]!r} (tol {tol[i[:-1] + (0,)]!r})")


def max_rel(a, b):
    """max over rows of |a - b|_inf / |b|_inf."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.max(np.abs(a - b), -1) / np.maximum(np.max(np.abs(b), -1), 1e-30)))


def elementwise_rel(a, b, floor_frac=1e-2):
    """max over elements of |a - b| / max(|b|, floor_frac * max|b_row|): the
    element-relative error, with elements far below their row's magnitude
    (where only absolute error is meaningful) measured against that floor."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.maximum(np.abs(b), floor_frac * np.max(np.abs(b), axis=-1, keepdims=True))
    return float(np.max(np.abs(a - b) / np.maximum(den, 1e-300)))


def report(a, b, what):
    """Prints the row-relative and element-relative errors of a vs b."""
    print(f"{what}: row-relative {max_rel(a, b):.2e}, element-relative {elementwise_rel(a, b):.2e}")
