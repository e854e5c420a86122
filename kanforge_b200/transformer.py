"""KAN feed-forward block of a transformer (reference kanforge/torch/transformer.py:25-52)."""

from __future__ import annotations

import torch
from torch import nn

from .layers import GRKAN, KANLinear


class KANFFN(nn.Module):
    """dim -> hidden -> dim with GR-KAN layers (``kind="grkan"``, KAT: the first
    rational starts as the identity, the second as ``activation``) or KANLinear."""

    def __init__(self, dim: int, hidden: int | None = None, kind: str = "grkan", basis="bspline", groups: int = 8,
                 activation: str = "gelu", dropout: float = 0.0, **kan_kwargs):
        super().__init__()
        hidden = hidden or 4 * dim
        if kind == "grkan":
            self.fc1 = GRKAN(dim, hidden, groups=groups, init="identity", **kan_kwargs)
            self.fc2 = GRKAN(hidden, dim, groups=groups, init=activation, **kan_kwargs)
        elif kind == "kan":
            self.fc1 = KANLinear(dim, hidden, basis, **kan_kwargs)
            self.fc2 = KANLinear(hidden, dim, basis, **kan_kwargs)
        else:
            raise ValueError("kind must be 'grkan' or 'kan'")
        self.drop = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.drop(self.fc2(self.drop(self.fc1(x))))
