"""Equivariant normalisation (flash_eq/layers/norm.py in the reference, :19-249).

Node-level work with the reference's parameter names: ``RepNorm`` (per-irrep norms),
``EquivariantLayerNorm`` (LayerNorm over the multiplicity of the irrep norms),
``SeparableEquivariantLayerNorm`` (LayerNorm over channels for l = 0, one shared RMS for
all l > 0 with a per-channel scale).  On CUDA float32 inputs with autograd not tracking,
each runs as one native kernel (csrc/feq_node.cu, one warp per node); under autograd the
PyTorch formulation below (the reference's) is used so that gradients flow.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..representations import Repr
from ..utils import get_epsilon


def native_node_ok(x: torch.Tensor, *params) -> bool:
    """True when the native node kernel may run: CUDA float32 and nothing for autograd to track."""
    if not (torch.is_tensor(x) and x.is_cuda and x.dtype == torch.float32 and x.dim() >= 2):
        return False
    if torch.is_grad_enabled() and (x.requires_grad or any(p is not None and p.requires_grad for p in params)):
        return False
    return True


class RepNorm(nn.Module):
    """Norm of every irrep component: (..., dim) -> (..., nreps)."""

    def __init__(self, repr: Repr, epsilon: float | None = None) -> None:
        super().__init__()
        self.num_reps = repr.nreps()
        self._epsilon = epsilon
        self._lvals = tuple(repr.lvals.tolist())
        self.register_buffer("indices", torch.tensor(repr.indices(), dtype=torch.long))

    def forward(self, st: torch.Tensor) -> torch.Tensor:
        eps = self._epsilon if self._epsilon is not None else get_epsilon(st.dtype)
        if native_node_ok(st) and st.shape[-1] == len(self.indices):
            from ..cuda import ops

            return ops.node_rep_norm(st, self._lvals, eps)
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
        self._lvals = tuple(repr.lvals.tolist())

    def forward(self, f: torch.Tensor) -> torch.Tensor:
        eps = self._epsilon if self._epsilon is not None else get_epsilon(f.dtype)
        ln = self.lnorm
        if native_node_ok(f, *(() if ln is None else (ln.weight, ln.bias))) and f.shape[-2] == self.mult:
            from ..cuda import ops

            rep_eps = self.norm._epsilon if self.norm._epsilon is not None else get_epsilon(f.dtype)
            return ops.node_layernorm(f, self._lvals, None if ln is None else ln.weight,
                                      None if ln is None else ln.bias, 0.0 if ln is None else ln.eps, rep_eps, eps)
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
        # device index vectors (not in the state dict): indexing with them needs no host sync
        self.register_buffer("_scalar_ix", torch.tensor(self.scalar_locs, dtype=torch.long), persistent=False)
        self.register_buffer("_higher_ix", torch.nonzero(mask).flatten(), persistent=False)
        self.nhigher = repr.nreps() - self.nscalar
        if self.nscalar > 0:
            self.scalar_norm = _ChannelLayerNorm(repr.mult, self.nscalar, epsilon)
        if self.nhigher > 0:
            self.higher_norm = _EquivariantRMSNorm(repr.mult, epsilon)

    def forward(self, f: torch.Tensor) -> torch.Tensor:
        sn = self.scalar_norm if self.nscalar > 0 else None
        hn = self.higher_norm if self.nhigher > 0 else None
        params = (() if sn is None else (sn.weight, sn.bias)) + (() if hn is None else (hn.weight,))
        if native_node_ok(f, *params) and f.shape[-2] == self.repr.mult:
            from ..cuda import ops

            eps_of = lambda m: m._epsilon if m._epsilon is not None else get_epsilon(f.dtype)
            eps = eps_of(sn) if sn is not None else eps_of(hn)
            return ops.node_sep_layernorm(f, tuple(self.repr.lvals.tolist()), None if sn is None else sn.weight,
                                          None if sn is None else sn.bias, None if hn is None else hn.weight, eps)
        out = f.clone()
        if self.nscalar > 0:
            out[..., self._scalar_ix] = self.scalar_norm(f[..., self._scalar_ix])
        if self.nhigher > 0:
            out[..., self._higher_ix] = self.higher_norm(f[..., self._higher_ix])
        return out

    def extra_repr(self) -> str:
        return f"nscalar={self.nscalar}, nhigher={self.nhigher}"
