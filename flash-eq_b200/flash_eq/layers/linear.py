"""SO(3)-equivariant linear layers (flash_eq/layers/linear.py in the reference).

``EquivariantEdgewiseLinear`` computes out = Q . Lambda(r) . P^T . f per edge in
one native call (rotate into the edge frame, distance-interpolated block-diagonal
mix, rotate back).  The reference does bmm -> block_diagonal_cuda -> bmm with
argsort/gather copies around the kernel (linear.py:100-160).

When P and Q are the unmodified outputs of ``WignerDBasis`` (or ``LazyBasis``
handles) for the same directions, the kernel rebuilds their blocks from the
directions and never reads the dense matrices; any other P / Q is applied as a
dense matrix exactly like the reference's bmm.

``EquivariantLinear`` (linear.py:172-268) is node-level: on the inference path native
position-major layout kernels (csrc/feq_node.cu) around one library GEMM per irrep; under
autograd one batched GEMM over positions.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..cuda import ops
from ..cuda.block_diagonal import block_diagonal_cuda, forward_only
from ..representations import ProductRepr, Repr
from ..representations.wigner import LazyBasis, basis_source
from .norm import native_node_ok
from .radial import SeparableRadialNet


DEFAULT_MIX_PRECISION = "bf16x3"
# Highest degree, per mix mode, for which the layer takes the one-kernel separable path on the
# GPU (lvals [0..L], mult 64).  Measured on a B200 at 640 000 edges of the config-2 graph, the
# one-kernel path against the binned three-kernel pipeline: bf16x3 L <= 2 1.49 / 2.38 ms,
# L = 3 4.41 / 8.36 ms, L = 4 6.18 / 7.32 ms; bf16 L = 3 4.09 / 7.41 ms, but L = 4 6.03 /
# 5.05 ms, so bf16 at L = 4 stays on the binned pipeline.
SEPARABLE_MAX_L = {"bf16x3": 4, "bf16": 3}


def _dense(M):
    return M.dense() if isinstance(M, LazyBasis) else M


class EquivariantEdgewiseLinear(nn.Module):
    """Edgewise equivariant linear map with distance-binned radial weights."""

    radial_weights: SeparableRadialNet

    def __init__(self, in_repr: Repr, out_repr: Repr, num_bins: int = 100, rank: int = 4, hidden_dim: int = 64,
                 min_dist: float = 0.0, max_dist: float = 10.0, log_bins: bool = False,
                 solid_harmonic_scale: float = 0.1) -> None:
        super().__init__()
        self.in_repr, self.out_repr = in_repr, out_repr
        self.rank = rank
        self.solid_harmonic_scale = solid_harmonic_scale
        self.product_repr = ProductRepr(in_repr, out_repr)
        self.weight_dim = self.product_repr.nreps()
        self.channels_in, self.channels_out = in_repr.mult, out_repr.mult
        self.radial_weights = SeparableRadialNet(num_bins=num_bins, out_mult=self.channels_out,
                                                 in_mult=self.channels_in, weight_dim=self.weight_dim, rank=rank,
                                                 hidden_dim=hidden_dim, min_val=min_dist, max_val=max_dist,
                                                 log=log_bins)
        self._lin = tuple(in_repr.lvals.tolist())
        self._lout = tuple(out_repr.lvals.tolist())
        # Arithmetic of the radial mix (not a reference kwarg, so not in __init__):
        # "fp32" CUDA-core float32, "bf16x3" tensor cores at float32-level accuracy,
        # "bf16" tensor cores with bf16 operands (the bf16-mix mode).
        self.mix_precision = DEFAULT_MIX_PRECISION

    def forward(self, P, Q, edge_features: torch.Tensor, distances: torch.Tensor) -> torch.Tensor:
        """(E, Cin, d_in) edge features -> (E, Cout, d_out), standard SH order."""
        return self._run(P, Q, edge_features, distances)

    def _run(self, P, Q, x, distances, src=None, edge_add=None):
        rw = self.radial_weights
        E = distances.shape[0]
        if E == 0:
            return torch.zeros(0, self.channels_out, self.out_repr.dim(), device=x.device, dtype=x.dtype)
        p1, p2 = rw.binning_params()
        dist = distances.to(torch.float32)
        grad = torch.is_grad_enabled() and (
            any(t is not None and t.requires_grad for t in (x, dist, edge_add, P if torch.is_tensor(P) else None,
                                                            Q if torch.is_tensor(Q) else None))
            or any(p.requires_grad for p in rw.parameters()))
        dP, dQ = basis_source(P, self._lin), basis_source(Q, self._lout)
        fused = dP is not None and dQ is not None and dP is dQ
        if not grad and fused and self._separable_ok(x):
            # the table is never formed: one kernel interpolates the radial features per
            # edge and applies the channel patterns on the tensor cores
            with torch.no_grad():
                feats = rw.radial_features()
            return ops.edgewise_separable_fwd(
                x.detach(), dist.detach(), rw.channel_patterns.detach(), feats, self._lin, self._lout,
                self.solid_harmonic_scale, p1, p2, rw.num_bins, rw.log, directions=dP, src=src,
                edge_add=None if edge_add is None else edge_add.detach(), mix=self.mix_precision)
        table = rw()
        if grad:
            return self._run_autograd(P, Q, x, dist, table, p1, p2, src, edge_add)
        Pd = Qd = None
        if not fused:
            Pd, Qd = _dense(P), _dense(Q)

        def run(xx, tab, dd, ea, pp, qq):
            return ops.edgewise_fwd(
                xx.detach(), dd.detach(), tab.detach(), self._lin, self._lout, self.channels_out,
                self.solid_harmonic_scale, p1, p2, rw.num_bins, rw.log, src=src,
                edge_add=None if ea is None else ea.detach(), directions=dP if fused else None,
                P=None if pp is None else pp.detach(), Q=None if qq is None else qq.detach(),
                mix=self.mix_precision)

        return forward_only(run, x, table, dist, edge_add, Pd, Qd)

    def _separable_ok(self, x) -> bool:
        """Whether the one-kernel separable path serves this call (layer shape, mix and a
        CUDA float32 input); cached per mix mode."""
        if not (x.is_cuda and x.dtype == torch.float32):
            return False
        if max(self._lin + self._lout) > SEPARABLE_MAX_L.get(self.mix_precision, -1):
            return False
        key = self.mix_precision
        cache = self.__dict__.setdefault("_sep_cache", {})
        if key not in cache:
            cache[key] = ops.separable_supported(self._lin, self._lout, self.channels_in, self.channels_out,
                                                 self.rank, key)
        return cache[key]

    def _run_autograd(self, P, Q, x, dist, table, p1, p2, src, edge_add):
        """The reference's three steps (linear.py:135-160) with autograd: bmm into the edge
        frame, block_diagonal_cuda (native forward and backward), bmm back out."""
        for M in (P, Q):
            d = M.directions if isinstance(M, LazyBasis) else None
            if d is not None and d.requires_grad:
                raise NotImplementedError("flash-eq B200: gradients with respect to edge directions are not "
                                          "supported (the Wigner basis is computed without autograd)")
        f = x[src] if src is not None else x
        if edge_add is not None:
            f = f + edge_add
        f_diag = torch.bmm(f, _dense(P))
        out_diag = block_diagonal_cuda(f_diag, table, dist, self.product_repr, p1, p2, self.radial_weights.num_bins,
                                       self.radial_weights.log, self.solid_harmonic_scale, mix=self.mix_precision)
        return torch.bmm(out_diag, _dense(Q).mT)

    def extra_repr(self) -> str:
        rw = self.radial_weights
        return (f"in_repr={self.in_repr}, out_repr={self.out_repr}, num_bins={rw.num_bins}, "
                f"dist=[{rw.min_val}, {rw.max_val}], spacing={'log' if rw.log else 'linear'}, rank={self.rank}")


class EquivariantLinear(nn.Module):
    """Per-degree channel mixing; bias (and activation) on l = 0 components only."""

    def __init__(self, in_repr: Repr, out_repr: Repr, bias: bool = True, activation: nn.Module | None = None) -> None:
        super().__init__()
        if not torch.equal(in_repr.lvals, out_repr.lvals):
            raise ValueError(
                "EquivariantLinear cannot modify the degrees of a representation. "
                f"Got input lvals={in_repr.lvals.tolist()}, output lvals={out_repr.lvals.tolist()}"
            )
        self.in_repr, self.out_repr = in_repr, out_repr
        self.weight = nn.Parameter(torch.empty(in_repr.nreps() * out_repr.mult, in_repr.mult))
        nn.init.xavier_uniform_(self.weight)
        self.register_buffer("indices", torch.tensor(in_repr.indices(), dtype=torch.long))
        self.expanddims = (1, out_repr.mult, in_repr.dim())
        self.outdims = (in_repr.nreps(), out_repr.mult, in_repr.dim())
        nscalar, self.scalar_locs = in_repr.find_scalar()
        self.register_buffer("_scalar_ix", torch.tensor(self.scalar_locs, dtype=torch.long), persistent=False)
        self.bias: nn.Parameter | None
        self.bias = nn.Parameter(torch.zeros(out_repr.mult, nscalar)) if (nscalar > 0 and bias) else None
        self.activation = activation if activation is not None else nn.Identity()
        self._lvals = tuple(in_repr.lvals.tolist())
        # inference path: position-major layout kernels around one GEMM per irrep (identity activation)
        self._native_ok = (isinstance(self.activation, nn.Identity) and in_repr.mult % 4 == 0
                           and out_repr.mult % 4 == 0)
        pos_ix = torch.full((in_repr.dim(),), -1, dtype=torch.int8)
        for s_i, loc in enumerate(self.scalar_locs):
            pos_ix[loc] = s_i
        self.register_buffer("_pos_scalar_ix", pos_ix, persistent=False)

    def forward(self, f: torch.Tensor) -> torch.Tensor:
        """out[..., co, p] = sum_ci W_{irrep(p)}[co, ci] f[..., ci, p] (+ bias on l = 0 positions).

        The reference forms (weight @ f) for every irrep at every position and gathers the
        matching one (linear.py:230-268).  Here the rows of each position's own irrep are
        gathered first and one batched GEMM over positions does only the needed products:
        the same sums, 1 / nreps of the FLOPs, no (nreps x) intermediate."""
        *b, cin, d = f.shape
        nreps = self.outdims[0]
        cout = self.expanddims[1]
        if self._native_ok and native_node_ok(f, self.weight, self.bias):
            return ops.node_linear(f, self._lvals, self.weight, self.bias, cout, self._pos_scalar_ix)
        x = f.reshape(-1, cin, d)
        w = self.weight.view(nreps, cout, cin).index_select(0, self.indices)    # (d, Cout, Cin)
        y = torch.bmm(w, x.permute(2, 1, 0))                                     # (d, Cout, N)
        if self.bias is not None:
            ys = y.index_select(0, self._scalar_ix) + self.bias.t().unsqueeze(-1)
            y = y.index_copy(0, self._scalar_ix, self.activation(ys).to(y.dtype))
        return y.permute(2, 1, 0).reshape(*b, cout, d)
