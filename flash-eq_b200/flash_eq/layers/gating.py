"""Norm-based gating (flash_eq/layers/gating.py:17-76 in the reference); node-level PyTorch."""
from __future__ import annotations

import torch
import torch.nn as nn

from ..representations import Repr
from ..utils import init_linear_weights
from .norm import RepNorm


class EquivariantGating(nn.Module):
    """x * sigmoid(Linear(irrep norms)) broadcast over each irrep's components."""

    def __init__(self, repr: Repr) -> None:
        super().__init__()
        self.repr = repr
        self.norm = RepNorm(repr)
        n = repr.nreps() * repr.mult
        self.linear = nn.Linear(n, n)
        self.register_buffer("ix", torch.tensor(repr.indices(), dtype=torch.long))
        self.outdims = (repr.mult, repr.nreps())
        self.activation = nn.Sigmoid()
        self.apply(init_linear_weights)

    def forward(self, st: torch.Tensor) -> torch.Tensor:
        norms = self.norm(st)
        *b, _, _ = norms.size()
        g = self.activation(self.linear(norms.flatten(-2, -1)).view(*b, *self.outdims))
        return st * g[..., self.ix]
