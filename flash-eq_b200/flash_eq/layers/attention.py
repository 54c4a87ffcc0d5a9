"""Equivariant graph attention (flash_eq/layers/attention.py in the reference).

``EquivariantEdgeAttention``: logits = scale * <Q, K> per head (minus d / decay),
softmax over the edges that share a destination, V weighted per head
(attention.py:72-167).  The softmax is one native segment kernel over the
graph's dst-sorted segments (the reference: scatter amax, gather, exp,
scatter_add, gather, divide).

``EquivariantAttention`` (attention.py:271-314): node-level norm + Q/K
projection in PyTorch; V = fused gather (x[src] + edge features) + edgewise
linear in one native call; then one fused native kernel computes the logits
from Q[dst] and K[src], the online softmax and the weighted pooling onto each
destination, without materialising Q[dst], K[src] or the weighted edges.

Under autograd every operator here has a native backward
(``flash_eq.cuda.attention_autograd``): gradients reach Q/K (and through them the
norm and projection), V (and the edgewise linear), log_scale and the distances.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..cuda import attention_autograd as aag
from ..cuda import ops
from ..graph import Graph
from ..partition import PartitionedGraph
from ..representations import Repr
from .linear import EquivariantEdgewiseLinear, EquivariantLinear
from .norm import EquivariantLayerNorm
from .pooling import GraphPooling, pool_edges


class _ScalarCache:
    """Host copy of a scalar parameter, refreshed only when the parameter changes
    (avoids a device->host sync per forward)."""

    def __init__(self):
        self._key = None
        self._val = 0.0

    def get(self, p: torch.Tensor, fn) -> float:
        key = (p.data_ptr(), p._version, p.device)
        if key != self._key:
            self._val = float(fn(p.detach()).item())
            self._key = key
        return self._val


class EquivariantEdgeAttention(nn.Module):
    """Scaled dot-product attention over each destination's in-edges."""

    def __init__(self, num_heads: int, qk_dim: int, dropout: float = 0.0,
                 distance_decay_scale: float | None = None) -> None:
        super().__init__()
        self.num_heads, self.qk_dim = num_heads, qk_dim
        self.distance_decay_scale = distance_decay_scale
        self.log_scale = nn.Parameter(torch.tensor(qk_dim ** -0.5).log())
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self._scale_cache = _ScalarCache()

    @property
    def scale(self) -> torch.Tensor:
        return self.log_scale.exp()

    def _scale_value(self) -> float:
        return self._scale_cache.get(self.log_scale, torch.exp)

    def _neighbor_softmax(self, logits: torch.Tensor, dst_indices: torch.Tensor, num_nodes: int) -> torch.Tensor:
        """Softmax of (E, H) logits over edges sharing a destination (attention.py:108-141)."""
        perm, offsets, status = ops.edge_sort(dst_indices, num_nodes)
        if int(status.item()) != 0:
            raise ValueError("dst_indices has indices outside [0, num_nodes)")
        return aag.segment_softmax(logits, perm, offsets, num_nodes)

    def attention_weights(self, Q, K, graph: Graph, distances=None) -> torch.Tensor:
        """(E, H) softmax weights of the logits scale * <Q, K> (- d / decay); differentiable in
        Q, K, distances and log_scale."""
        decay = self.distance_decay_scale if distances is not None else None
        return aag.edge_attention_weights(Q, K, distances, self.log_scale, graph, self._scale_value(), decay)

    def forward(self, Q, K, V, graph: Graph, distances: torch.Tensor | None = None) -> torch.Tensor:
        w = self.dropout(self.attention_weights(Q, K, graph, distances))
        return self._apply_attention(V, w)

    def _apply_attention(self, V: torch.Tensor, attn_weights: torch.Tensor) -> torch.Tensor:
        E, mult, dim = V.shape
        if self.num_heads == 1:
            return V * attn_weights.view(E, 1, 1)
        hd = mult // self.num_heads
        return (V.view(E, self.num_heads, hd, dim) * attn_weights.view(E, self.num_heads, 1, 1)).view(E, mult, dim)

    def extra_repr(self) -> str:
        return f"num_heads={self.num_heads}, qk_dim={self.qk_dim}"


class EquivariantAttention(nn.Module):
    """Equivariant attention layer: Q/K projection, edgewise V, softmax, pooling."""

    def __init__(self, in_repr: Repr, out_repr: Repr, num_heads: int = 1, num_bins: int = 100, rank: int = 4,
                 hidden_dim: int = 64, min_dist: float = 0.0, max_dist: float = 10.0, log_bins: bool = False,
                 dropout: float = 0.0, reduce: str = "sum", distance_decay_scale: float | None = None) -> None:
        super().__init__()
        if in_repr.mult % num_heads != 0:
            raise ValueError(f"num_heads ({num_heads}) must divide in_repr.mult ({in_repr.mult})")
        if out_repr.mult % num_heads != 0:
            raise ValueError(f"num_heads ({num_heads}) must divide out_repr.mult ({out_repr.mult})")
        self.in_repr, self.out_repr, self.num_heads = in_repr, out_repr, num_heads
        self.norm_qk = EquivariantLayerNorm(in_repr)
        self.linear_qk = EquivariantLinear(in_repr, Repr(lvals=in_repr.lvals, mult=in_repr.mult * 2), bias=False)
        self.attention = EquivariantEdgeAttention(num_heads=num_heads,
                                                  qk_dim=(in_repr.mult // num_heads) * in_repr.dim(),
                                                  dropout=dropout, distance_decay_scale=distance_decay_scale)
        self.linear_v = EquivariantEdgewiseLinear(in_repr, out_repr, num_bins=num_bins, rank=rank,
                                                  hidden_dim=hidden_dim, min_dist=min_dist, max_dist=max_dist,
                                                  log_bins=log_bins)
        self.pool = GraphPooling(reduce=reduce)

    def forward(self, P, Q_basis, node_features: torch.Tensor, distances: torch.Tensor, graph: Graph,
                edge_features: torch.Tensor | None = None) -> torch.Tensor:
        """(N, Cin, d_in) node features -> (N, Cout, d_out)."""
        mult = self.in_repr.mult
        qk = self.linear_qk(self.norm_qk(node_features))        # (N, 2C, d) node level
        k_src = None
        x_src = node_features
        if isinstance(graph, PartitionedGraph):
            # src rows live on other ranks: per layer one halo exchange of the inputs and one of K
            # (all_to_all_single of just the rows this rank's edges read)
            x_src = graph.gather_nodes(node_features)
            k_src = graph.gather_nodes(qk[:, mult:].contiguous())
        V = self.linear_v._run(P, Q_basis, x_src, distances, src=graph.src, edge_add=edge_features)
        att = self.attention
        dropping = self.training and isinstance(att.dropout, nn.Dropout)
        if self.pool.reduce in ("sum", "mean") and not dropping:
            decay = att.distance_decay_scale
            scale = att._scale_value()
            if k_src is not None:
                return aag.attn_pool(qk[:, :mult].contiguous(), V, distances, att.log_scale, graph, self.num_heads,
                                     scale, decay, self.pool.reduce, k=k_src)
            return aag.attn_pool(qk, V, distances, att.log_scale, graph, self.num_heads, scale, decay,
                                 self.pool.reduce)
        # max pooling or attention dropout: materialise per-edge weights
        E = graph.num_edges
        Qe = qk[:, :mult][graph.dst].reshape(E, self.num_heads, -1)
        Ke = (qk[:, mult:] if k_src is None else k_src)[graph.src].reshape(E, self.num_heads, -1)
        w = att.dropout(att.attention_weights(Qe, Ke, graph, distances))
        return pool_edges(V, graph, self.pool.reduce, weights=w)

    def extra_repr(self) -> str:
        return (f"in_repr={self.in_repr}, out_repr={self.out_repr}, num_heads={self.num_heads}, "
                f"reduce='{self.pool.reduce}'")
