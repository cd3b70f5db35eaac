"""manifold_b200: the recurrent geodesic-flow (leapfrog) hot path of the
reference package ``gfn`` (Manifold-Laboratory/manifold), re-built for
NVIDIA B200 (sm_100a).  ``import manifold_b200 as gfn`` exposes the
reference's model / layer / integrator / geometry / scan API for that path.
"""
__version__ = "0.1.0"

from . import _lib
from ._lib import GfnError
from .model import Manifold, ImplicitReadout
from .model import Manifold as GFN
from .layers import MLayer, ParallelMLayer, RiemannianGating
from .layers import MLayer as GLayer
from .geometry import LowRankChristoffel, ReactiveChristoffel, ToroidalChristoffel
from .integrators import (DormandPrinceIntegrator, EulerIntegrator, ForestRuthIntegrator,
                          HeunIntegrator, LeapfrogIntegrator, OmelyanIntegrator, RK4Integrator,
                          SymplecticIntegrator, VerletIntegrator, YoshidaIntegrator)
from .integrators import INTEGRATOR_CLASSES as INTEGRATORS
from .embeddings import FunctionalEmbedding, ImplicitEmbedding, SineLayer
from .scan import parallel_scan
from .losses import CrossEntropyLoss, cross_entropy
from . import cuda

__all__ = ["CrossEntropyLoss", "cross_entropy", "GFN", "Manifold", "GLayer", "MLayer", "ParallelMLayer", "RiemannianGating",
           "LowRankChristoffel", "ReactiveChristoffel", "ToroidalChristoffel", "LeapfrogIntegrator",
           "EulerIntegrator", "HeunIntegrator", "RK4Integrator", "DormandPrinceIntegrator",
           "SymplecticIntegrator", "VerletIntegrator", "YoshidaIntegrator", "ForestRuthIntegrator",
           "OmelyanIntegrator",
           "FunctionalEmbedding", "ImplicitEmbedding", "SineLayer", "ImplicitReadout",
           "parallel_scan", "GfnError", "INTEGRATORS"]
