"""Equivariant transformer blocks (flash_eq/layers/transformer.py in the reference).

Same structure and parameter names: pre-norm attention with a LayerScale'd
residual (only when in_repr == out_repr), pre-norm gated MLP with residual
(transformer.py:66-260), and the stack that builds the edge geometry and one
shared basis (transformer.py:263-437).  The stack passes ``LazyBasis`` handles to
its blocks, so per-edge P / Q matrices are never materialised: the edgewise
kernel rebuilds their blocks from the edge vectors.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..graph import Graph
from ..partition import PartitionedGraph
from ..representations import Repr, WignerDBasis
from .attention import EquivariantAttention
from .gating import EquivariantGating
from .linear import EquivariantLinear
from .norm import SeparableEquivariantLayerNorm


class LayerScale(nn.Module):
    """x * gamma with a learnable scalar gamma (CaiT)."""

    def __init__(self, init_value: float = 1e-4) -> None:
        super().__init__()
        self.gamma = nn.Parameter(torch.tensor(init_value))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x * self.gamma


class DropPath(nn.Module):
    """Stochastic depth: in training, drop the whole sublayer with probability p."""

    def __init__(self, drop_prob: float = 0.0) -> None:
        super().__init__()
        self.drop_prob = drop_prob

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.drop_prob == 0.0 or not self.training:
            return x
        if torch.rand(1, device=x.device).item() < self.drop_prob:
            return torch.zeros_like(x)
        return x / (1 - self.drop_prob)


class EquivariantTransformerBlock(nn.Module):
    """norm -> attention (+ residual) -> norm -> gated MLP (+ residual)."""

    def __init__(self, in_repr: Repr, out_repr: Repr, num_heads: int = 1, num_bins: int = 100, rank: int = 4,
                 hidden_dim: int = 64, min_dist: float = 0.0, max_dist: float = 10.0, log_bins: bool = False,
                 mlp_ratio: int = 2, dropout: float = 0.0, drop_path: float = 0.0,
                 layer_scale_init: float | None = 1e-4, use_gating: bool = True, use_s2_activation: bool = False,
                 s2_precision: int = 47, distance_decay_scale: float | None = None) -> None:
        super().__init__()
        if use_s2_activation:
            raise NotImplementedError(
                "use_s2_activation=True (the S^2 / Lebedev activation) is not part of flash-eq B200; "
                "the default gated MLP is.")
        self.in_repr, self.out_repr = in_repr, out_repr
        self.use_s2_activation = use_s2_activation
        self._use_attn_residual = torch.equal(in_repr.lvals, out_repr.lvals) and in_repr.mult == out_repr.mult
        self.norm1 = SeparableEquivariantLayerNorm(in_repr)
        self.attn = EquivariantAttention(in_repr=in_repr, out_repr=out_repr, num_heads=num_heads, num_bins=num_bins,
                                         rank=rank, hidden_dim=hidden_dim, min_dist=min_dist, max_dist=max_dist,
                                         log_bins=log_bins, dropout=dropout, reduce="sum",
                                         distance_decay_scale=distance_decay_scale)
        self.norm2 = SeparableEquivariantLayerNorm(out_repr)
        hidden = Repr(lvals=out_repr.lvals, mult=out_repr.mult * mlp_ratio)
        self.mlp_up = EquivariantLinear(out_repr, hidden, bias=True)
        self.mlp_act: nn.Module = EquivariantGating(hidden) if use_gating else nn.Identity()
        self.mlp_down = EquivariantLinear(hidden, out_repr, bias=True)
        self.layer_scale_attn = (LayerScale(layer_scale_init) if layer_scale_init is not None
                                 and self._use_attn_residual else nn.Identity())
        self.layer_scale_mlp = LayerScale(layer_scale_init) if layer_scale_init is not None else nn.Identity()
        self.drop_path = DropPath(drop_path) if drop_path > 0.0 else nn.Identity()

    def _residual(self, x: torch.Tensor, y: torch.Tensor, scale: nn.Module) -> torch.Tensor:
        """x + drop_path(scale(y)); with LayerScale and no stochastic depth in effect, one
        fused x + y * gamma (torch.addcmul) instead of a multiply and an add."""
        if isinstance(scale, LayerScale) and isinstance(self.drop_path, nn.Identity):
            return torch.addcmul(x, y, scale.gamma)
        return x + self.drop_path(scale(y))

    def forward(self, P, Q, node_features: torch.Tensor, distances: torch.Tensor, graph: Graph,
                edge_features: torch.Tensor | None = None) -> torch.Tensor:
        attn_out = self.attn(P, Q, self.norm1(node_features), distances, graph, edge_features=edge_features)
        if self._use_attn_residual:
            x = self._residual(node_features, attn_out, self.layer_scale_attn)
        else:
            x = attn_out
        mlp_out = self.mlp_down(self.mlp_act(self.mlp_up(self.norm2(x))))
        return self._residual(x, mlp_out, self.layer_scale_mlp)

    def extra_repr(self) -> str:
        return f"in_repr={self.in_repr}, out_repr={self.out_repr}, attn_residual={self._use_attn_residual}"


class EquivariantTransformer(nn.Module):
    """Stack of blocks: in_repr -> hidden_repr ... -> out_repr, with a final norm."""

    def __init__(self, in_repr: Repr, hidden_repr: Repr, out_repr: Repr, num_layers: int = 6, num_heads: int = 1,
                 num_bins: int = 100, rank: int = 4, hidden_dim: int = 64, min_dist: float = 0.0,
                 max_dist: float = 10.0, log_bins: bool = False, mlp_ratio: int = 2, dropout: float = 0.0,
                 drop_path: float = 0.0, layer_scale_init: float | None = 1e-4, use_s2_activation: bool = False,
                 s2_precision: int = 47, distance_decay_scale: float | None = None) -> None:
        super().__init__()
        self.in_repr, self.hidden_repr, self.out_repr = in_repr, hidden_repr, out_repr
        self.num_layers = num_layers
        self.distance_decay_scale = distance_decay_scale
        self._basis_reprs = [in_repr, hidden_repr, out_repr]
        self.basis = WignerDBasis(self._basis_reprs)
        rates = [x.item() for x in torch.linspace(0, drop_path, num_layers)]
        self.layers = nn.ModuleList()
        for i in range(num_layers):
            lin = in_repr if i == 0 else hidden_repr
            lout = out_repr if i == num_layers - 1 else hidden_repr
            self.layers.append(EquivariantTransformerBlock(
                in_repr=lin, out_repr=lout, num_heads=num_heads, num_bins=num_bins, rank=rank,
                hidden_dim=hidden_dim, min_dist=min_dist, max_dist=max_dist, log_bins=log_bins,
                mlp_ratio=mlp_ratio, dropout=dropout, drop_path=rates[i], layer_scale_init=layer_scale_init,
                use_s2_activation=use_s2_activation, s2_precision=s2_precision,
                distance_decay_scale=distance_decay_scale))
        self.final_norm = SeparableEquivariantLayerNorm(out_repr)

    def forward(self, coordinates: torch.Tensor, node_features: torch.Tensor, graph: Graph) -> torch.Tensor:
        if isinstance(graph, PartitionedGraph):      # src / dst are not global node ids there
            edge_vectors = graph.edge_vectors(coordinates)
        else:
            edge_vectors = coordinates[graph.src] - coordinates[graph.dst]    # src - dst (transformer.py:406)
        distances = edge_vectors.norm(dim=-1)
        m_in, m_hidden, m_out = self.basis.lazy(edge_vectors)
        x = node_features
        for i, layer in enumerate(self.layers):
            P = m_in if i == 0 else m_hidden
            Q = m_out if i == self.num_layers - 1 else m_hidden
            x = layer(P, Q, x, distances, graph)
        return self.final_norm(x)

    def extra_repr(self) -> str:
        return (f"in_repr={self.in_repr}, hidden_repr={self.hidden_repr}, out_repr={self.out_repr}, "
                f"num_layers={self.num_layers}")
