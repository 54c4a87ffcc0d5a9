"""Irreducible representations of SO(3) and their bookkeeping.

Behaviour follows flash_eq/representations/types.py:30-350 of the reference:
``Irrep`` (degree l, dim 2l+1, so(3) generators in the real spherical-harmonic
basis ordered [Lz, Lx, Ly]), ``ProductIrrep``, ``Repr`` (lvals, mult, dim,
cumdims, indices, l_indices, find_scalar) and ``ProductRepr`` (nreps = weight
dimension of the block-diagonal radial table).  The generator construction has
to agree with the reference's convention exactly, since every basis matrix is
derived from it; it is evaluated here in float64 with numpy and rounded to
float32 at the end, like the reference's REAL_DTYPE.
"""
from __future__ import annotations

from typing import Any, Generator, List, Sequence

import numpy as np
import torch


def _real_so3_generators(l: int) -> np.ndarray:
    """[Lz, Lx, Ly] for degree l in the real SH basis (float64).

    J+/J- ladder operators in the complex |l, m> basis, Jx, Jy, Jz from them,
    then conjugation by the complex->real change of basis Q; the real parts of
    Q^H Jy Q, Q^H Jx Q, Q^H Jz Q are returned in that order.
    """
    n = 2 * l + 1
    m = np.arange(-l, l + 1)
    jp = np.zeros((n, n), dtype=np.complex128)
    jm = np.zeros((n, n), dtype=np.complex128)
    for i in range(n - 1):
        jp[i + 1, i] = -np.sqrt(l * (l + 1) - m[i] * (m[i] + 1))
        jm[i, i + 1] = np.sqrt(l * (l + 1) - m[i + 1] * (m[i + 1] - 1))
    jx = 0.5 * (jp + jm)
    jy = -0.5j * (jp - jm)
    jz = 1j * np.diag(m.astype(np.complex128))
    q = _complex_to_real(l)
    qh = q.conj().T
    return np.stack([(qh @ jy @ q).real, (qh @ jx @ q).real, (qh @ jz @ q).real])


def _complex_to_real(l: int) -> np.ndarray:
    n = 2 * l + 1
    r = 2 ** -0.5
    q = np.zeros((n, n), dtype=np.complex128)
    for k in range(1, l + 1):
        sign = (-1) ** k
        q[l - k, l + k] = r
        q[l - k, l - k] = -1j * r
        q[l + k, l + k] = sign * r
        q[l + k, l - k] = 1j * sign * r
    q[l, l] = 1.0
    return ((-1j) ** l) * q


class Irrep:
    """Real irreducible representation of SO(3) of degree l (dimension 2l+1)."""

    REAL_DTYPE = torch.float32
    COMPLEX_DTYPE = torch.complex128

    def __init__(self, l: int, mult: int = 1) -> None:
        if not isinstance(l, int) or l < 0:
            raise ValueError(f"Degree l must be a non-negative integer, got {l}")
        if not isinstance(mult, int) or mult < 1:
            raise ValueError(f"Multiplicity must be a positive integer, got {mult}")
        self.l = l
        self.mult = mult

    def __eq__(self, other: Any) -> bool:
        return isinstance(other, Irrep) and (self.l, self.mult) == (other.l, other.mult)

    def __hash__(self) -> int:
        return hash((self.l, self.mult))

    def dim(self) -> int:
        return 2 * self.l + 1

    def mvals(self) -> torch.Tensor:
        return torch.arange(-self.l, self.l + 1)

    def raising(self) -> torch.Tensor:
        m = torch.arange(-self.l, self.l)
        return torch.diag(-torch.sqrt(self.l * (self.l + 1) - m * (m + 1)), diagonal=-1)

    def lowering(self) -> torch.Tensor:
        m = torch.arange(-self.l + 1, self.l + 1)
        return torch.diag(torch.sqrt(self.l * (self.l + 1) - m * (m - 1)), diagonal=1)

    def _generators(self) -> torch.Tensor:
        """(3, 2l+1, 2l+1) generators [Lz, Lx, Ly], float32."""
        return torch.from_numpy(_real_so3_generators(self.l)).to(self.REAL_DTYPE)

    def toreal(self) -> torch.Tensor:
        return torch.from_numpy(_complex_to_real(self.l))

    def __str__(self) -> str:
        return f"Irrep(l={self.l}, mult={self.mult})"


class ProductIrrep:
    """Decomposition of irrep1 x irrep2 into degrees |l1-l2| .. l1+l2."""

    def __init__(self, rep1: Irrep, rep2: Irrep) -> None:
        self.rep1, self.rep2 = rep1, rep2
        self.lmin = abs(rep1.l - rep2.l)
        self.lmax = rep1.l + rep2.l
        self.reps = [Irrep(l) for l in range(self.lmin, self.lmax + 1)]

    def dim(self) -> int:
        return sum(r.dim() for r in self.reps)

    def maxdim(self) -> int:
        return max(r.dim() for r in self.reps)

    def nreps(self) -> int:
        return len(self.reps)

    def __str__(self) -> str:
        return f"ProductIrrep({self.rep1.l} x {self.rep2.l})"


class Repr:
    """A list of irreps sharing one multiplicity."""

    def __init__(self, lvals: Sequence[int], mult: int = 1) -> None:
        if not hasattr(lvals, "__len__"):
            raise TypeError(f"lvals must be a sequence, got {type(lvals).__name__}")
        if len(lvals) == 0:
            raise ValueError("lvals must contain at least one degree")
        if not isinstance(mult, int) or mult < 1:
            raise ValueError(f"Multiplicity must be a positive integer, got {mult}")
        self.irreps = [Irrep(int(l), mult) for l in lvals]
        self.lvals = torch.tensor([ir.l for ir in self.irreps], dtype=torch.long)
        self.mult = mult
        dims = [ir.dim() for ir in self.irreps]
        self._cumdims = torch.tensor([0] + list(np.cumsum(dims)), dtype=torch.long)

    def nreps(self) -> int:
        return len(self.irreps)

    def __iter__(self) -> Generator[Irrep, None, None]:
        yield from self.irreps

    def __eq__(self, other: Any) -> bool:
        return isinstance(other, Repr) and torch.equal(self.lvals, other.lvals) and self.mult == other.mult

    def __hash__(self) -> int:
        return hash((tuple(self.lvals.tolist()), self.mult))

    def dim(self) -> int:
        return sum(ir.dim() for ir in self.irreps)

    def lmax(self) -> int:
        return max(ir.l for ir in self.irreps)

    def cumdims(self) -> torch.Tensor:
        return self._cumdims

    def mvals(self) -> torch.Tensor:
        return torch.cat([ir.mvals() for ir in self.irreps])

    def indices(self) -> List[int]:
        out: List[int] = []
        for i, ir in enumerate(self.irreps):
            out += [i] * ir.dim()
        return out

    def l_indices(self) -> torch.Tensor:
        return self.lvals[self.indices()]

    def find_scalar(self) -> tuple[int, List[int]]:
        locs, off = [], 0
        for ir in self.irreps:
            if ir.l == 0:
                locs.append(off)
            off += ir.dim()
        return len(locs), locs

    def __str__(self) -> str:
        return "Repr(lvals=[" + ", ".join(str(ir.l) for ir in self.irreps) + "])"


class ProductRepr:
    """Tensor product of two representations; nreps() is the radial-table weight dim."""

    def __init__(self, rep1: Repr, rep2: Repr) -> None:
        self.rep1, self.rep2 = rep1, rep2
        self.reps = [ProductIrrep(a, b) for a in rep1 for b in rep2]

    def dim(self) -> int:
        return sum(r.dim() for r in self.reps)

    def __eq__(self, other: Any) -> bool:
        return isinstance(other, ProductRepr) and self.rep1 == other.rep1 and self.rep2 == other.rep2

    def __hash__(self) -> int:
        return hash((hash(self.rep1), hash(self.rep2)))

    def lmax(self) -> int:
        return max(r.lmax for r in self.reps)

    def nreps(self) -> int:
        return sum(r.nreps() for r in self.reps)

    def __str__(self) -> str:
        return f"ProductRepr({self.rep1} x {self.rep2})"
