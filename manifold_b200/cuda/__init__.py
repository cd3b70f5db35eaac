"""B200 kernels behind the reference's ``gfn.cuda`` operator boundary."""
from .ops import christoffel_fused, leapfrog_fused  # noqa: F401

__all__ = ["christoffel_fused", "leapfrog_fused"]
