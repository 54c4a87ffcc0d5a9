"""Wigner-D matrices and the per-edge basis (flash_eq/representations/wigner.py
in the reference: random_rotation :27-93, WignerD :96-240, the m-first
permutation :243-272, WignerDBasis :275-374).

``WignerDBasis.forward`` runs the native basis kernel: each (edge, degree) block
is a closed form in the edge's polar angles instead of a batched
``torch.linalg.matrix_exp`` of the whole (dim x dim) generator.  The returned
dense matrices match the reference's (m-first column order).  Each returned
tensor also carries a small provenance tag; when it reaches
``EquivariantEdgewiseLinear`` unmodified, the fused kernel rebuilds the blocks
from the directions in shared memory instead of reading the dense matrix.
``LazyBasis`` goes one step further and never materialises the matrix.
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.nn as nn

from ..utils import get_epsilon
from .types import Repr


def random_rotation(shape: tuple[int, ...] = (), device=None, dtype: torch.dtype = torch.float32):
    """Haar-uniform rotations as (axis (*shape, 3), angle (*shape,)), from unit quaternions."""
    q = torch.randn((*shape, 4), device=device, dtype=dtype)
    q = q / q.norm(dim=-1, keepdim=True)
    sign = torch.sign(q[..., 0:1])
    q = q * torch.where(sign == 0, torch.ones_like(sign), sign)
    half = torch.acos(q[..., 0].clamp(-1.0, 1.0))
    angle = 2 * half
    s = torch.sin(half)
    small = s < 1e-6
    axis = q[..., 1:] / torch.where(small, torch.ones_like(s), s)[..., None]
    ez = torch.zeros_like(axis)
    ez[..., 2] = 1.0
    axis = torch.where(small[..., None], ez, axis)
    axis = axis / (axis.norm(dim=-1, keepdim=True) + 1e-8)
    return axis, angle


def _build_m_order_permutation(lvals: torch.Tensor) -> torch.Tensor:
    """Standard (l, m) order -> m-first order: all m=0 entries (one per irrep), then
    for m = 1..lmax and each irrep with l >= m the pair (+m, -m)."""
    lv = [int(x) for x in lvals]
    offs, o = [], 0
    for l in lv:
        offs.append(o)
        o += 2 * l + 1
    perm = [offs[i] + l for i, l in enumerate(lv)]
    for m in range(1, (max(lv) if lv else 0) + 1):
        for i, l in enumerate(lv):
            if l >= m:
                perm += [offs[i] + l + m, offs[i] + l - m]
    return torch.tensor(perm, dtype=torch.long)


class _BasisTag:
    """Provenance of a basis tensor: which directions and lvals produced it."""

    __slots__ = ("directions", "dir_version", "lvals", "out_version")

    def __init__(self, directions, lvals, out):
        self.directions = directions
        self.dir_version = directions._version
        self.lvals = tuple(int(x) for x in lvals)
        self.out_version = out._version


def basis_source(M, lvals):
    """Directions (E, 3) that generated basis ``M`` for ``lvals``, or None if ``M`` is
    an arbitrary / modified matrix (then the dense matrix is used as given)."""
    if isinstance(M, LazyBasis):
        return M.directions if M.lvals == tuple(int(x) for x in lvals) else None
    tag = getattr(M, "_feq_basis", None)
    if tag is None or tag.lvals != tuple(int(x) for x in lvals):
        return None
    if M._version != tag.out_version or tag.directions._version != tag.dir_version:
        return None
    return tag.directions


class LazyBasis:
    """A basis that is never materialised: (directions, lvals).  Accepted wherever
    this package's layers take P / Q; ``dense()`` builds the matrix on demand."""

    def __init__(self, directions: torch.Tensor, lvals):
        self.directions = directions
        self.lvals = tuple(int(x) for x in lvals)

    @property
    def shape(self):
        d = sum(2 * l + 1 for l in self.lvals)
        return torch.Size((self.directions.shape[0], d, d))

    def dense(self) -> torch.Tensor:
        from ..cuda import ops

        M = ops.wigner_basis(self.directions, self.lvals)
        M._feq_basis = _BasisTag(self.directions, self.lvals, M)
        return M


def _as_directions(directions: torch.Tensor) -> torch.Tensor:
    if not directions.is_cuda:
        from ..cuda.ops import CUDANotAvailableError

        if not torch.cuda.is_available():
            raise CUDANotAvailableError("flash-eq requires a CUDA-capable GPU. No CUDA device was detected.")
        raise RuntimeError("flash-eq B200 computes Wigner-D bases on the GPU; move the directions to CUDA")
    if directions.dtype != torch.float32:
        raise TypeError(f"flash-eq B200 computes in float32; got directions of dtype {directions.dtype}")
    return directions.detach().contiguous()


class WignerD(nn.Module):
    """Wigner D-matrices of a representation."""

    def __init__(self, repr: Repr) -> None:
        super().__init__()
        self.repr = repr
        dim = repr.dim()
        gens = torch.zeros(3, dim, dim)
        for i, ir in enumerate(repr.irreps):
            a, b = int(repr.cumdims()[i]), int(repr.cumdims()[i + 1])
            gens[:, a:b, a:b] = ir._generators()
        self.register_buffer("generators", gens.view(3, -1))

    def _apply(self, fn, *args, **kwargs):
        super()._apply(fn, *args, **kwargs)
        if self.generators.dtype == torch.float16:   # matrix_exp is unusable in fp16
            self.generators = self.generators.float()
        return self

    def rot(self, axis: torch.Tensor, angle: torch.Tensor, cartesian: bool = False) -> torch.Tensor:
        """D = exp(angle * (axis . G)), G ordered [Lz, Lx, Ly] (cartesian=True reorders a
        Cartesian axis to [z, x, y]).  General-axis utility (not the edge hot path)."""
        if cartesian:
            axis = axis[..., [2, 0, 1]]
        dim = self.repr.dim()
        *b, _ = axis.size()
        in_dtype = axis.dtype
        if in_dtype == torch.float16:
            axis, angle = axis.float(), angle.float()
        K = angle[..., None, None] * (axis @ self.generators.to(axis.dtype)).view(*b, dim, dim)
        r = torch.nan_to_num(torch.linalg.matrix_exp(K), 0.0)
        if in_dtype == torch.float16:
            r = r.half()
        cd = self.repr.cumdims()
        for i, ir in enumerate(self.repr.irreps):
            if ir.l == 0:
                r[..., cd[i], cd[i]] = 1.0
        return r

    def rot_to_ez(self, directions: torch.Tensor, cartesian: bool = False) -> torch.Tensor:
        """D(g_x^-1) for the rotation taking e_z to each direction (native kernel)."""
        if cartesian:
            raise NotImplementedError("rot_to_ez(cartesian=True) is not part of the edge path")
        from ..cuda import _lib, ops

        d = _as_directions(directions)
        flat = d.reshape(-1, 3)
        out = ops.wigner_basis(flat, self.repr.lvals.tolist(), _lib.FEQ_BASIS_ROT_TO_EZ)
        return out.view(*d.shape[:-1], out.shape[-2], out.shape[-1])


class WignerDBasis(nn.Module):
    """Per-edge basis matrices for a list of representations (deduplicated by lvals)."""

    def __init__(self, reprs: Sequence[Repr]) -> None:
        super().__init__()
        if len(reprs) == 0:
            raise ValueError("reprs must contain at least one Repr")
        self.reprs = list(reprs)
        seen: dict[tuple[int, ...], int] = {}
        self._input_to_unique: list[int] = []
        unique: list[Repr] = []
        for r in reprs:
            key = tuple(r.lvals.tolist())
            if key not in seen:
                seen[key] = len(unique)
                unique.append(r)
            self._input_to_unique.append(seen[key])
        self._num_unique = len(unique)
        self._unique_lvals = [tuple(r.lvals.tolist()) for r in unique]
        self._wigner_modules = nn.ModuleList([WignerD(r) for r in unique])
        for i, r in enumerate(unique):
            self.register_buffer(f"_perm_{i}", _build_m_order_permutation(r.lvals))

    def forward(self, directions: torch.Tensor) -> tuple[torch.Tensor, ...]:
        """directions (E, 3) -> one (E, dim, dim) matrix per input Repr (m-first columns)."""
        from ..cuda import ops

        d = _as_directions(directions)
        mats = []
        for lv in self._unique_lvals:
            M = ops.wigner_basis(d, lv)
            M._feq_basis = _BasisTag(d, lv, M)
            mats.append(M)
        return tuple(mats[i] for i in self._input_to_unique)

    def lazy(self, directions: torch.Tensor) -> tuple[LazyBasis, ...]:
        """Same as forward but returns unmaterialised ``LazyBasis`` handles."""
        d = _as_directions(directions)
        return tuple(LazyBasis(d, self._unique_lvals[i]) for i in self._input_to_unique)

    def extra_repr(self) -> str:
        return f"reprs=[{', '.join(str(r) for r in self.reprs)}], num_unique={self._num_unique}"
