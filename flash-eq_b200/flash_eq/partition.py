"""Destination-range partition of one graph across ranks (one process per GPU).

No counterpart in the reference, which runs a graph on one device.  Rank r owns the
contiguous node range [starts[r], starts[r+1]) — boundaries chosen on the cumulative
in-degree so every rank holds about E / world_size edges — and every edge whose dst it
owns.  Softmax, pooling and the edgewise mix of an edge then only need the src-side
node rows.  A rank's edges read its own rows plus a halo: the other ranks' nodes that
are the src of one of its edges.  Once per attention layer the halo rows are exchanged
with one NCCL ``all_to_all_single`` (each owner sends exactly the rows each peer reads),
and ``src`` indexes the array [owned rows; halo rows] (halo in global node order).  Every
rank holds the whole graph, so every rank derives every rank's halo locally and the
exchange plan needs no communication.

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
    """The edges of one rank: ``src`` indexes [owned rows; halo rows] (``num_src_nodes``
    rows), ``dst`` the rank's own rows; ``num_nodes`` is the number of owned rows.
    Exchange plan: ``send_idx`` lists the owned rows the peers read, grouped by peer
    (``send_counts``); ``recv_counts[r]`` halo rows come from rank r."""
    num_src_nodes: int = 0
    node_start: int = 0
    node_end: int = 0
    world_size: int = 1
    rank: int = 0
    src_global: torch.Tensor | None = None
    dst_global: torch.Tensor | None = None
    edge_ids: torch.Tensor | None = None
    halo_global: torch.Tensor | None = None
    send_idx: torch.Tensor | None = None
    send_counts: list = field(default_factory=list)
    recv_counts: list = field(default_factory=list)
    group: object = field(default=None, repr=False, compare=False)

    def __post_init__(self) -> None:
        if self.src.dim() != 1 or self.dst.dim() != 1 or self.src.shape[0] != self.dst.shape[0]:
            raise ValueError("src and dst must be 1D tensors of the same length")
        if self.num_nodes < 0 or self.num_src_nodes < 0 or self.num_src_nodes < self.num_nodes:
            raise ValueError(f"bad partition sizes: {self.num_nodes} owned rows, {self.num_src_nodes} source rows")

    def _key(self):
        return super()._key() + (self.num_src_nodes,)

    def _check_src(self):
        return ((self.src < 0) | (self.src >= self.num_src_nodes)).any() if self.num_edges else None

    def _num_src_rows(self) -> int:
        return self.num_src_nodes

    @property
    def num_halo(self) -> int:
        return self.num_src_nodes - self.num_nodes

    def to(self, device) -> "PartitionedGraph":
        mv = lambda t: None if t is None else t.to(device)
        return PartitionedGraph(src=self.src.to(device), dst=self.dst.to(device), num_nodes=self.num_nodes,
                                num_src_nodes=self.num_src_nodes, node_start=self.node_start,
                                node_end=self.node_end, world_size=self.world_size, rank=self.rank,
                                src_global=mv(self.src_global), dst_global=mv(self.dst_global),
                                edge_ids=mv(self.edge_ids), halo_global=mv(self.halo_global),
                                send_idx=mv(self.send_idx), send_counts=list(self.send_counts),
                                recv_counts=list(self.recv_counts), group=self.group)

    def edge_vectors(self, coordinates: torch.Tensor) -> torch.Tensor:
        """coordinates[src] - coordinates[dst] with global node ids (coordinates: (N, 3))."""
        return coordinates[self.src_global] - coordinates[self.dst_global]

    def gather_nodes(self, owned: torch.Tensor) -> torch.Tensor:
        """Owned rows (num_nodes, ...) -> [owned rows; halo rows] (num_src_nodes, ...).

        Differentiable: the backward returns each halo row's gradient to its owner (the
        reverse exchange) and adds it, peer by peer in rank order, onto the owned rows."""
        if owned.shape[0] != self.num_nodes:
            raise ValueError(f"expected {self.num_nodes} owned rows, got {owned.shape[0]}")
        if self.world_size == 1:
            return owned.contiguous()
        if torch.is_grad_enabled() and owned.requires_grad:
            return _GatherNodes.apply(owned, self)
        return self._forward_exchange(owned.detach())

    def _forward_exchange(self, owned: torch.Tensor) -> torch.Tensor:
        owned = owned.contiguous()
        send = owned.index_select(0, self.send_idx)
        halo = _exchange(send, self.send_counts, self.recv_counts, self.group)
        return torch.cat([owned, halo])


# Exchange timing (no counterpart in the reference): when set to a list, every exchange
# appends a (start, end) pair of CUDA events recorded on the current stream around its
# collective; benchmarks read the elapsed times after synchronising.
EXCHANGE_EVENTS: list | None = None


def _exchange(send: torch.Tensor, send_counts, recv_counts, group) -> torch.Tensor:
    """Rows send[...] split by ``send_counts`` go to ranks 0..W-1; returns the rows received,
    split by ``recv_counts`` in rank order.  One ``all_to_all_single`` on every backend (NCCL
    on the GPUs, gloo in the host tests): a collective, so a peer that has left ends it with
    an error (gloo) or a process-group timeout (NCCL) instead of a wait without end."""
    import torch.distributed as dist

    recv = send.new_empty((int(sum(recv_counts)),) + tuple(send.shape[1:]))
    ev = None
    if EXCHANGE_EVENTS is not None and send.is_cuda:
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
    dist.all_to_all_single(recv, send.contiguous(), output_split_sizes=list(recv_counts),
                           input_split_sizes=list(send_counts), group=group)
    if ev is not None:
        ev[1].record()
        EXCHANGE_EVENTS.append(ev)
    return recv


class _GatherNodes(torch.autograd.Function):
    @staticmethod
    def forward(ctx, owned, part):
        ctx.part = part
        return part._forward_exchange(owned)

    @staticmethod
    def backward(ctx, grad):
        part = ctx.part
        grad = grad.contiguous()
        mine = grad[: part.num_nodes].clone()
        back = _exchange(grad[part.num_nodes:].contiguous(), part.recv_counts, part.send_counts, part.group)
        off = 0
        for c in part.send_counts:                 # fixed order: bitwise reproducible sums
            if c:
                mine.index_add_(0, part.send_idx[off:off + c], back[off:off + c])
            off += c
        return mine, None


def partition_graph(graph: Graph, world_size: int, rank: int, group=None) -> PartitionedGraph:
    """This rank's part of a dst-range partition of ``graph`` (same result on every rank)."""
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside [0, {world_size})")
    N = graph.num_nodes
    dev = graph.src.device
    bounds = dst_range_bounds(graph.dst, N, world_size).to(dev)
    start, end = int(bounds[rank]), int(bounds[rank + 1])
    dst = graph.dst.to(torch.int64)
    src = graph.src.to(torch.int64)
    own_e = torch.searchsorted(bounds[1:], dst, right=True)       # rank holding each edge
    own_s = torch.searchsorted(bounds[1:], src, right=True)       # rank owning its src row
    # every rank's halo: unique (reader, node) pairs with a src owned elsewhere, sorted by
    # reader, then node id (so each reader's halo is grouped by owner, in rank order)
    cross = own_s != own_e
    pairs = torch.unique(own_e[cross] * max(N, 1) + src[cross])
    reader, node = pairs // max(N, 1), pairs % max(N, 1)
    node_owner = torch.searchsorted(bounds[1:], node, right=True)
    halo = node[reader == rank]
    recv_counts = torch.bincount(node_owner[reader == rank], minlength=world_size).tolist()
    sent = node_owner == rank
    send_idx = node[sent] - start
    send_counts = torch.bincount(reader[sent], minlength=world_size).tolist()
    # this rank's edges, original edge order kept
    eids = torch.nonzero(own_e == rank, as_tuple=False).flatten()
    s_g, d_g = src[eids], dst[eids]
    local = (s_g >= start) & (s_g < end)
    s_loc = torch.where(local, s_g - start, (end - start) + torch.searchsorted(halo, s_g))
    return PartitionedGraph(src=s_loc, dst=d_g - start, num_nodes=end - start,
                            num_src_nodes=(end - start) + int(halo.shape[0]), node_start=start, node_end=end,
                            world_size=world_size, rank=rank, src_global=s_g, dst_global=d_g, edge_ids=eids,
                            halo_global=halo, send_idx=send_idx, send_counts=send_counts,
                            recv_counts=recv_counts, group=group)
