"""The feed-forward block of a KAN transformer (reference kanforge/torch/transformer.py:25-52).

``KANFFN(dim, hidden, kind, ...)`` maps dim -> hidden -> dim with two KAN
layers and dropout after each:

* ``kind="grkan"``: KAT's two group-rational layers, the first rational
  starting as the identity and the second as ``activation`` (their linear
  maps run on the GR-KAN tensor-core kernels for bf16, on the three-TF32
  GEMM for float32); ``kan_kwargs`` do not apply to them, as in the reference;
* ``kind="kan"``: two KANLinear layers of ``basis`` with ``kan_kwargs``.
"""

from __future__ import annotations

import torch
from torch import nn

from .layers import GRKAN, KANLinear

FFN_KINDS = ("grkan", "kan")


def _ffn_layers(kind: str, dim: int, hidden: int, basis, groups: int, activation: str, kan_kwargs: dict):
    if kind == "grkan":
        return (GRKAN(dim, hidden, groups=groups, init="identity"), GRKAN(hidden, dim, groups=groups, init=activation))
    if kind == "kan":
        return KANLinear(dim, hidden, basis, **kan_kwargs), KANLinear(hidden, dim, basis, **kan_kwargs)
    raise ValueError("kind must be 'grkan' or 'kan'")


class KANFFN(nn.Module):
    """dim -> hidden (default 4 dim) -> dim with KAN layers; attributes ``fc1``,
    ``fc2`` and ``drop`` as in the reference, so state dicts carry over."""

    def __init__(self, dim: int, hidden: int | None = None, kind: str = "grkan", basis="bspline", groups: int = 8,
                 activation: str = "gelu", dropout: float = 0.0, **kan_kwargs):
        super().__init__()
        self.fc1, self.fc2 = _ffn_layers(kind, dim, hidden or 4 * dim, basis, groups, activation, kan_kwargs)
        self.drop = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.drop(self.fc1(x))
        return self.drop(self.fc2(h))
