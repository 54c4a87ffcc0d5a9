"""Destination-range partition of one graph across ranks (one process per GPU).

No counterpart in the reference, which runs a graph on one device.  Rank r owns the
contiguous node range [starts[r], starts[r+1]) — boundaries chosen on the cumulative
in-degree so every rank holds about E / world_size edges — and every edge whose dst it
owns.  Softmax, pooling and the edgewise mix of an edge then only need the src-side
node rows; those are exchanged once per attention layer with one NCCL
``all_gather_into_tensor`` of each rank's owned rows (padded to a common row count, so
the gathered array is indexed by ``rank * rows_per_rank + local row``).

    part = partition_graph(graph, world_size, rank, group)
    y_owned = model(coordinates, x[part.node_start:part.node_end], part)

``coordinates`` stay global (N, 3); ``node_features`` and the output are the owned rows.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .graph import Graph


def dst_range_bounds(dst: torch.Tensor, num_nodes: int, world_size: int) -> torch.Tensor:
    """Node boundaries (world_size + 1,) splitting the in-edges into ~equal contiguous parts."""
    if world_size < 1:
        raise ValueError(f"world_size must be >= 1, got {world_size}")
    deg = torch.bincount(dst.to(torch.int64).cpu(), minlength=num_nodes)
    cum = torch.cumsum(deg, 0)
    E = int(cum[-1]) if num_nodes else 0
    targets = torch.tensor([E * r / world_size for r in range(1, world_size)], dtype=torch.float64)
    inner = torch.searchsorted(cum.to(torch.float64), targets, right=False) + 1
    bounds = torch.cat([torch.zeros(1, dtype=torch.int64), inner.clamp(0, num_nodes),
                        torch.full((1,), num_nodes, dtype=torch.int64)])
    return torch.cummax(bounds, 0).values


@dataclass
class PartitionedGraph(Graph):
    """The edges of one rank: ``src`` indexes the gathered (padded) node array, ``dst`` the
    rank's own rows; ``num_nodes`` is the number of owned rows."""
    num_src_nodes: int = 0
    node_start: int = 0
    node_end: int = 0
    rows_per_rank: int = 0
    world_size: int = 1
    rank: int = 0
    src_global: torch.Tensor | None = None
    dst_global: torch.Tensor | None = None
    edge_ids: torch.Tensor | None = None
    group: object = field(default=None, repr=False, compare=False)

    def __post_init__(self) -> None:
        if self.src.dim() != 1 or self.dst.dim() != 1 or self.src.shape[0] != self.dst.shape[0]:
            raise ValueError("src and dst must be 1D tensors of the same length")
        if self.num_nodes < 0 or self.num_src_nodes < 1:
            raise ValueError(f"bad partition sizes: {self.num_nodes} owned rows, {self.num_src_nodes} source rows")

    def _key(self):
        return super()._key() + (self.num_src_nodes,)

    def _check_src(self):
        return ((self.src < 0) | (self.src >= self.num_src_nodes)).any() if self.num_edges else None

    def _num_src_rows(self) -> int:
        return self.num_src_nodes

    def to(self, device) -> "PartitionedGraph":
        mv = lambda t: None if t is None else t.to(device)
        return PartitionedGraph(src=self.src.to(device), dst=self.dst.to(device), num_nodes=self.num_nodes,
                                num_src_nodes=self.num_src_nodes, node_start=self.node_start,
                                node_end=self.node_end, rows_per_rank=self.rows_per_rank,
                                world_size=self.world_size, rank=self.rank, src_global=mv(self.src_global),
                                dst_global=mv(self.dst_global), edge_ids=mv(self.edge_ids), group=self.group)

    def edge_vectors(self, coordinates: torch.Tensor) -> torch.Tensor:
        """coordinates[src] - coordinates[dst] with global node ids (coordinates: (N, 3))."""
        return coordinates[self.src_global] - coordinates[self.dst_global]

    def gather_nodes(self, owned: torch.Tensor) -> torch.Tensor:
        """All ranks' owned rows (num_nodes, ...) -> (world_size * rows_per_rank, ...).

        Differentiable: the backward sums every rank's gradient of the gathered array
        (a reduce-scatter) and keeps this rank's owned rows."""
        if owned.shape[0] != self.num_nodes:
            raise ValueError(f"expected {self.num_nodes} owned rows, got {owned.shape[0]}")
        if self.world_size == 1:
            return owned.contiguous()
        if torch.is_grad_enabled() and owned.requires_grad:
            return _GatherNodes.apply(owned, self)
        return self._all_gather(owned.detach())

    def _all_gather(self, owned: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        pad = owned.new_zeros((self.rows_per_rank,) + tuple(owned.shape[1:]))
        pad[: owned.shape[0]] = owned
        if dist.get_backend(self.group) == "gloo":      # host-side runs (tests): list form
            parts = [torch.empty_like(pad) for _ in range(self.world_size)]
            dist.all_gather(parts, pad, group=self.group)
            return torch.cat(parts)
        out = owned.new_empty((self.world_size * self.rows_per_rank,) + tuple(owned.shape[1:]))
        dist.all_gather_into_tensor(out, pad, group=self.group)
        return out


class _GatherNodes(torch.autograd.Function):
    @staticmethod
    def forward(ctx, owned, part):
        ctx.part = part
        return part._all_gather(owned)

    @staticmethod
    def backward(ctx, grad):
        import torch.distributed as dist

        part = ctx.part
        rows = part.rows_per_rank
        grad = grad.contiguous()
        if dist.get_backend(part.group) == "gloo":      # host-side runs (tests): all-reduce, then slice
            total = grad.clone()
            dist.all_reduce(total, group=part.group)
            mine = total[part.rank * rows: part.rank * rows + part.num_nodes]
        else:
            out = grad.new_empty((rows,) + tuple(grad.shape[1:]))
            dist.reduce_scatter_tensor(out, grad, group=part.group)
            mine = out[: part.num_nodes]
        return mine.contiguous(), None


def partition_graph(graph: Graph, world_size: int, rank: int, group=None) -> PartitionedGraph:
    """This rank's part of a dst-range partition of ``graph`` (same result on every rank)."""
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside [0, {world_size})")
    N = graph.num_nodes
    bounds = dst_range_bounds(graph.dst, N, world_size).to(graph.src.device)
    counts = bounds[1:] - bounds[:-1]
    rows = max(1, int(counts.max()))
    start, end = int(bounds[rank]), int(bounds[rank + 1])
    dst = graph.dst.to(torch.int64)
    src = graph.src.to(torch.int64)
    mask = (dst >= start) & (dst < end)
    eids = torch.nonzero(mask, as_tuple=False).flatten()          # original edge order kept
    s_g, d_g = src[eids], dst[eids]
    owner = torch.searchsorted(bounds[1:], s_g, right=True)
    s_pad = owner * rows + (s_g - bounds[owner])
    return PartitionedGraph(src=s_pad, dst=d_g - start, num_nodes=end - start,
                            num_src_nodes=world_size * rows, node_start=start, node_end=end,
                            rows_per_rank=rows, world_size=world_size, rank=rank, src_global=s_g,
                            dst_global=d_g, edge_ids=eids, group=group)
