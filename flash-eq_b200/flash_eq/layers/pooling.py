"""Edge -> node pooling (flash_eq/layers/pooling.py:21-109 in the reference).

The reference uses scatter_add_ / scatter_reduce_ (atomics, order varies run to
run).  Here every node reduces its own in-edges in edge-id order through the
graph's dst-sorted segments: same values, deterministic.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..cuda import attention_autograd as aag
from ..graph import Graph

_REDUCES = ("sum", "mean", "max")


def pool_edges(edge_features: torch.Tensor, graph: Graph, reduce: str = "sum",
               weights: torch.Tensor | None = None) -> torch.Tensor:
    """(E, C, d) -> (N, C, d); optional per-head weights (E, H) multiply each head's channels.
    Differentiable in edge_features and weights (native backward)."""
    if reduce not in _REDUCES:
        raise ValueError(f"reduce must be one of {list(_REDUCES)}, got '{reduce}'")
    return aag.segment_pool(edge_features, graph, reduce, weights)


class GraphPooling(nn.Module):
    """Aggregate edge features onto destination nodes: 'sum', 'mean' or 'max'."""

    def __init__(self, reduce: str = "sum") -> None:
        super().__init__()
        if reduce not in _REDUCES:
            raise ValueError(f"reduce must be one of {list(_REDUCES)}, got '{reduce}'")
        self.reduce = reduce

    def forward(self, edge_features: torch.Tensor, graph: Graph) -> torch.Tensor:
        return pool_edges(edge_features, graph, self.reduce)

    def extra_repr(self) -> str:
        return f"reduce='{self.reduce}'"
