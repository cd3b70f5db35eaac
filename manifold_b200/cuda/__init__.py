"""B200 kernels behind the reference's ``gfn.cuda`` operator boundary."""
from .ops import (christoffel_backward, christoffel_fused, leapfrog_backward,  # noqa: F401
                  leapfrog_fused, reactive_christoffel, recurrent_manifold_fused)
from .autograd import christoffel_fused_autograd, leapfrog_fused_autograd  # noqa: F401

__all__ = ["christoffel_fused", "christoffel_backward", "reactive_christoffel", "leapfrog_fused",
           "leapfrog_backward", "recurrent_manifold_fused", "christoffel_fused_autograd",
           "leapfrog_fused_autograd"]
