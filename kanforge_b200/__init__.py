"""kanforge_b200 -- the KAN layer hot path of kanforge on B200 (sm_100a).

Drop-in for the reference's torch layers on CUDA:

    from kanforge_b200 import KAN, KANLinear, GRKAN, KANConv2d, KANFFN, Chebyshev
    layer = KANLinear(4096, 4096, Chebyshev(12), device="cuda", dtype=torch.bfloat16)

The forward and backward passes, the closed derivative primitives and
``edge_derivative`` run hand-written CUDA kernels from ``libkanb200.so``
(build with ``python -m kanforge_b200.build``).
"""

from . import bases, convert, kernels
from .bases import *  # noqa: F401,F403
from .bases import __all__ as _bases_all
from .conv import KANConv1d, KANConv2d, KANConv3d
from .convert import load, save
from .layers import GRKAN, KAN, KANLinear, layer_inputs, rebuild_kan
from .plan import KernelPlan, plan_for
from .transformer import KANFFN

__version__ = "0.1.0"

__all__ = [
    *_bases_all,
    "GRKAN",
    "KAN",
    "KANConv1d",
    "KANConv2d",
    "KANConv3d",
    "KANFFN",
    "KANLinear",
    "KernelPlan",
    "bases",
    "convert",
    "kernels",
    "layer_inputs",
    "load",
    "plan_for",
    "rebuild_kan",
    "save",
    "__version__",
]
