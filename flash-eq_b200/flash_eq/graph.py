"""COO graph container (flash_eq/graph.py:15-97 in the reference) plus a cached
dst-sorted view.

The segment kernels (softmax, pooling, attention) walk each destination's
in-edges through ``perm``/``offsets`` built by a stable GPU radix sort of
``dst``.  The view is built once per graph and reused by every layer; building
it also validates that ``src`` and ``dst`` index into ``num_nodes`` (the one
place a host synchronisation happens per graph).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class Graph:
    src: torch.Tensor
    dst: torch.Tensor
    num_nodes: int
    _csr: tuple | None = field(default=None, init=False, repr=False, compare=False)
    _src_csr: tuple | None = field(default=None, init=False, repr=False, compare=False)

    def __post_init__(self) -> None:
        if self.src.dim() != 1:
            raise ValueError(f"src must be 1D, got shape {self.src.shape}")
        if self.dst.dim() != 1:
            raise ValueError(f"dst must be 1D, got shape {self.dst.shape}")
        if self.src.shape[0] != self.dst.shape[0]:
            raise ValueError(
                f"src and dst must have same length, got {self.src.shape[0]} and {self.dst.shape[0]}"
            )
        if self.num_nodes <= 0:
            raise ValueError(f"num_nodes must be positive, got {self.num_nodes}")

    @property
    def num_edges(self) -> int:
        return self.src.shape[0]

    @property
    def device(self) -> torch.device:
        return self.src.device

    @property
    def dtype(self) -> torch.dtype:
        return self.src.dtype

    def to(self, device: torch.device | str) -> "Graph":
        return Graph(src=self.src.to(device), dst=self.dst.to(device), num_nodes=self.num_nodes)

    @staticmethod
    def random(num_nodes: int, num_edges: int, device: torch.device | str = "cpu") -> "Graph":
        """Random graph; self-loops and multi-edges allowed."""
        src = torch.randint(0, num_nodes, (num_edges,), device=device)
        dst = torch.randint(0, num_nodes, (num_edges,), device=device)
        return Graph(src=src, dst=dst, num_nodes=num_nodes)

    @staticmethod
    def knn(coordinates: torch.Tensor, k: int) -> "Graph":
        """k-nearest-neighbour graph on the GPU (no counterpart in the reference): edges
        src -> dst where src ranges over the k nearest other nodes of dst, grouped by dst."""
        from .cuda import ops

        nbr = ops.knn(coordinates, k)
        n = coordinates.shape[0]
        dst = torch.arange(n, device=coordinates.device).repeat_interleave(k)
        src = nbr.reshape(-1)
        keep = src >= 0
        if not bool(keep.all()):
            src, dst = src[keep], dst[keep]
        return Graph(src=src, dst=dst, num_nodes=n)

    @staticmethod
    def radius(coordinates: torch.Tensor, r: float, batch: torch.Tensor | None = None,
               loop: bool = False) -> "Graph":
        """Radius graph on the GPU (no counterpart in the reference): an edge src -> dst for
        every ordered pair of nodes of the same graph (``batch`` ids; None: one graph) closer
        than ``r``, in (src, dst) order; no self loops unless ``loop``."""
        from .cuda import ops

        src, dst = ops.radius_graph(coordinates, r, batch=batch, loop=loop)
        return Graph(src=src, dst=dst, num_nodes=coordinates.shape[0])

    # -- dst-sorted view ----------------------------------------------------
    def _check_src(self):
        """Device bool: some src index lies outside [0, num_nodes) (None without edges)."""
        return ((self.src < 0) | (self.src >= self.num_nodes)).any() if self.num_edges else None

    def _key(self):
        return (self.src.data_ptr(), self.src._version, self.dst.data_ptr(), self.dst._version,
                self.num_nodes, self.src.shape[0])

    def dst_segments(self):
        """(perm, offsets): in-edges of node n are perm[offsets[n]:offsets[n+1]], in edge-id order."""
        key = self._key()
        if self._csr is not None and self._csr[0] == key:
            return self._csr[1], self._csr[2]
        from .cuda import ops

        perm, offsets, status = ops.edge_sort(self.dst, self.num_nodes)
        bad_src = self._check_src()
        if int(status.item()) != 0:
            raise ValueError("graph.dst has indices outside [0, num_nodes)")
        if bad_src is not None and bool(bad_src):
            raise ValueError("graph.src has indices outside [0, num_nodes)")
        self._csr = (key, perm, offsets)
        return perm, offsets

    def _num_src_rows(self) -> int:
        return self.num_nodes

    def src_segments(self):
        """(perm, offsets): out-edges of source row m are perm[offsets[m]:offsets[m+1]], in edge-id
        order (used by the backward of the attention, which reduces over each source's edges)."""
        key = self._key()
        if self._src_csr is not None and self._src_csr[0] == key:
            return self._src_csr[1], self._src_csr[2]
        from .cuda import ops

        self.dst_segments()            # validates src / dst
        perm, offsets, _ = ops.edge_sort(self.src, self._num_src_rows())
        self._src_csr = (key, perm, offsets)
        return perm, offsets
