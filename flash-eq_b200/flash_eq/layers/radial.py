"""Radial weight networks (flash_eq/layers/radial.py in the reference).

``SeparableRadialNet`` produces the binned table (num_bins + 1, Cout, Cin, W)
consumed by the edgewise kernel:  W[b, o, i, w] = sum_k C_k[o, i] f_k(r_b, w),
f from a sinusoid x DimeNet-envelope basis at the bin edges through a small
SiLU MLP (radial.py:133-296).  It is O(num_bins) work: on the GPU without autograd the
features at the bin edges come from one native launch (feq_radial_features), otherwise
from the PyTorch modules; parameter names and shapes match the reference so state dicts
load.
``RadialBasisFunctions`` / ``RadialMLP`` are kept for API completeness.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..utils import get_epsilon, init_linear_weights


class RadialBasisFunctions(nn.Module):
    """Gaussian RBFs with learnable centres and widths."""

    def __init__(self, num_functions: int, r_min: float = 0.0, r_max: float = 10.0) -> None:
        super().__init__()
        self.num_functions = num_functions
        self.mu = nn.Parameter(torch.linspace(r_min, r_max, num_functions))
        self.sigma = nn.Parameter(torch.full((num_functions,), (r_max - r_min) / max(num_functions - 1, 1)))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() > 1 and x.size(-1) == 1:
            x = x.squeeze(-1)
        z = (x[..., None] - self.mu) / self.sigma.abs().clamp(min=get_epsilon(self.sigma.dtype))
        return torch.exp(-z ** 2)


class RadialMLP(nn.Module):
    """distance -> (N, out_mult, in_mult, num_basis) through RBF + SiLU MLP."""

    def __init__(self, hidden_dim: int, num_basis: int, in_mult: int, out_mult: int, num_layers: int = 2,
                 r_max: float = 10.0) -> None:
        super().__init__()
        self.num_basis, self.in_mult, self.out_mult = num_basis, in_mult, out_mult
        self.rbf = RadialBasisFunctions(hidden_dim, r_min=0.0, r_max=r_max)
        layers: list[nn.Module] = [nn.Linear(hidden_dim, hidden_dim), nn.SiLU()]
        for _ in range(num_layers - 1):
            layers += [nn.Linear(hidden_dim, hidden_dim), nn.SiLU()]
        layers.append(nn.Linear(hidden_dim, out_mult * in_mult * num_basis))
        self.mlp = nn.Sequential(*layers)
        self.apply(init_linear_weights)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.mlp(self.rbf(x)).view(x.size(0), self.out_mult, self.in_mult, self.num_basis)


class SeparableRadialNet(nn.Module):
    """Binned separable radial weights: table (num_bins + 1, out_mult, in_mult, weight_dim)."""

    bin_edges: torch.Tensor
    frequencies: torch.Tensor

    def __init__(self, num_bins: int = 100, out_mult: int = 16, in_mult: int = 16, weight_dim: int = 7,
                 rank: int = 4, num_freqs: int = 16, hidden_dim: int = 64, min_val: float = 0.0,
                 max_val: float = 10.0, log: bool = False) -> None:
        super().__init__()
        if log and min_val <= 0:
            raise ValueError("min_val must be > 0 for log spacing")
        self.num_bins, self.out_mult, self.in_mult = num_bins, out_mult, in_mult
        self.weight_dim, self.rank = weight_dim, rank
        self.min_val, self.max_val, self.log = min_val, max_val, log
        self.channel_patterns = nn.Parameter(torch.empty(rank, out_mult, in_mult))
        nn.init.xavier_uniform_(self.channel_patterns)
        self.register_buffer("frequencies", torch.arange(1, num_freqs + 1, dtype=torch.float32) * torch.pi)
        self.trunk = nn.Sequential(nn.Linear(2 * num_freqs, hidden_dim), nn.SiLU(),
                                   nn.Linear(hidden_dim, hidden_dim), nn.SiLU())
        self.head = nn.Linear(hidden_dim, rank * weight_dim)
        if log:
            # exponents taken in float32, as radial.py:191-198 does
            self.register_buffer("bin_edges", torch.logspace(torch.tensor(min_val).log10().item(),
                                                             torch.tensor(max_val).log10().item(),
                                                             num_bins + 1))
            self._log_min = torch.tensor(min_val).log().item()
            self._inv_log_range = 1.0 / torch.tensor(max_val / min_val).log().item()
        else:
            self.register_buffer("bin_edges", torch.linspace(min_val, max_val, num_bins + 1))
        self.apply(init_linear_weights)

    def _sinusoidal_basis(self, r: torch.Tensor) -> torch.Tensor:
        x = ((r - self.min_val) / (self.max_val - self.min_val)).clamp(0.0, 1.0)
        env = 1.0 - 10.0 * x ** 3 + 15.0 * x ** 4 - 6.0 * x ** 5   # p=5 envelope (DimeNet)
        ang = x.unsqueeze(-1) * self.frequencies
        return torch.cat([torch.sin(ang) * env.unsqueeze(-1), torch.cos(ang) * env.unsqueeze(-1)], dim=-1)

    def radial_features(self) -> torch.Tensor:
        """f_k(r_b, w) at the bin edges, (num_bins + 1, rank, weight_dim): the factor of the
        table that depends on distance (radial.py:259-267).  On the GPU without autograd one
        native launch (feq_radial_features) computes it; under autograd the PyTorch modules
        below do, so gradients reach the radial net."""
        if self._native_features_ok():
            from ..cuda import ops
            l1, l2 = self.trunk[0], self.trunk[2]
            f = ops.radial_features(self.bin_edges, self.min_val, self.max_val, self.frequencies, l1.weight,
                                    l1.bias, l2.weight, l2.bias, self.head.weight, self.head.bias)
        else:
            f = self.head(self.trunk(self._sinusoidal_basis(self.bin_edges)))
        return f.view(-1, self.rank, self.weight_dim)

    def _native_features_ok(self) -> bool:
        if torch.is_grad_enabled() or not self.bin_edges.is_cuda:
            return False
        from ..cuda import ops
        l1, l2 = self.trunk[0], self.trunk[2]
        return (self.bin_edges.dtype == torch.float32 and l1.weight.dtype == torch.float32
                and self.frequencies.numel() <= ops.RADIAL_MAX_FREQS and l1.out_features <= ops.RADIAL_MAX_HIDDEN
                and l2.out_features == l1.out_features)

    def forward(self) -> torch.Tensor:
        return torch.einsum("koi,bkw->boiw", self.channel_patterns, self.radial_features())

    def binning_params(self) -> tuple[float, float]:
        if self.log:
            return self._log_min, self._inv_log_range
        return self.min_val, self.num_bins / (self.max_val - self.min_val)

    def bin_indices(self, values: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        if self.log:
            x = (values.float().clamp(min=self.min_val).log() - self._log_min) * self._inv_log_range * self.num_bins
        else:
            x = (values.float() - self.min_val) * (self.num_bins / (self.max_val - self.min_val))
        x = x.clamp(0.0, self.num_bins)
        lo = x.floor().int().clamp(max=self.num_bins - 1)
        return lo, (x - lo.float()).clamp(0.0, 1.0)
