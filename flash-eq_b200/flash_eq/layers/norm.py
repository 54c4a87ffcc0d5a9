"""Equivariant normalisation (flash_eq/layers/norm.py in the reference, :19-249).

Node-level work; kept in PyTorch with the reference's parameter names:
``RepNorm`` (per-irrep norms), ``EquivariantLayerNorm`` (LayerNorm over the
multiplicity of the irrep norms), ``SeparableEquivariantLayerNorm`` (LayerNorm
over channels for l = 0, one shared RMS for all l > 0 with a per-channel scale).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..representations import Repr
from ..utils import get_epsilon


class RepNorm(nn.Module):
    """Norm of every irrep component: (..., dim) -> (..., nreps)."""

    def __init__(self, repr: Repr, epsilon: float | None = None) -> None:
        super().__init__()
        self.num_reps = repr.nreps()
        self._epsilon = epsilon
        self.register_buffer("indices", torch.tensor(repr.indices(), dtype=torch.long))

    def forward(self, st: torch.Tensor) -> torch.Tensor:
        eps = self._epsilon if self._epsilon is not None else get_epsilon(st.dtype)
        sq = st * st
        out = torch.zeros(*sq.shape[:-1], self.num_reps, device=sq.device, dtype=sq.dtype)
        out.scatter_add_(-1, self.indices.expand(sq.shape), sq)
        return (out + eps).sqrt()


class _ChannelLayerNorm(nn.Module):
    """LayerNorm over the channel axis (dim -2) for the scalar components."""

    def __init__(self, mult: int, nscalar: int, epsilon: float | None = None) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(mult, nscalar))
        self.bias = nn.Parameter(torch.zeros(mult, nscalar))
        self._epsilon = epsilon

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        eps = self._epsilon if self._epsilon is not None else get_epsilon(x.dtype)
        mu = x.mean(dim=-2, keepdim=True)
        sd = x.std(dim=-2, keepdim=True, unbiased=False)
        return (x - mu) / (sd + eps) * self.weight + self.bias


class _EquivariantRMSNorm(nn.Module):
    """One RMS over channels and components, per-channel learnable scale."""

    def __init__(self, mult: int, epsilon: float | None = None) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(mult))
        self._epsilon = epsilon

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        eps = self._epsilon if self._epsilon is not None else get_epsilon(x.dtype)
        rms = torch.sqrt((x ** 2).mean(dim=(-2, -1), keepdim=True) + eps)
        return x * (self.weight[..., None] / rms)


class EquivariantLayerNorm(nn.Module):
    """LayerNorm of the irrep norms across multiplicity, applied as a rescaling."""

    def __init__(self, repr: Repr, epsilon: float | None = None) -> None:
        super().__init__()
        self.mult = repr.mult
        self.norm = RepNorm(repr)
        self.lnorm = nn.LayerNorm(repr.mult) if repr.mult > 1 else None
        self._epsilon = epsilon
        self.register_buffer("ix", torch.tensor(repr.indices(), dtype=torch.long))

    def forward(self, f: torch.Tensor) -> torch.Tensor:
        eps = self._epsilon if self._epsilon is not None else get_epsilon(f.dtype)
        norms = self.norm(f)
        if self.lnorm is None:
            return f * (1.0 / (norms + eps))[..., self.ix]
        ln = self.lnorm(norms.transpose(-2, -1)).transpose(-2, -1)
        return f * (ln / (norms + eps))[..., self.ix]


class SeparableEquivariantLayerNorm(nn.Module):
    """Scalars: channel LayerNorm; higher degrees: a shared RMS (EquiformerV2 style)."""

    def __init__(self, repr: Repr, epsilon: float | None = None) -> None:
        super().__init__()
        self.repr = repr
        self.nscalar, self.scalar_locs = repr.find_scalar()
        mask = torch.ones(repr.dim(), dtype=torch.bool)
        mask[self.scalar_locs] = False
        self.register_buffer("higher_mask", mask)
        self.nhigher = repr.nreps() - self.nscalar
        if self.nscalar > 0:
            self.scalar_norm = _ChannelLayerNorm(repr.mult, self.nscalar, epsilon)
        if self.nhigher > 0:
            self.higher_norm = _EquivariantRMSNorm(repr.mult, epsilon)

    def forward(self, f: torch.Tensor) -> torch.Tensor:
        out = f.clone()
        if self.nscalar > 0:
            out[..., self.scalar_locs] = self.scalar_norm(f[..., self.scalar_locs])
        if self.nhigher > 0:
            out[..., self.higher_mask] = self.higher_norm(f[..., self.higher_mask])
        return out

    def extra_repr(self) -> str:
        return f"nscalar={self.nscalar}, nhigher={self.nhigher}"
