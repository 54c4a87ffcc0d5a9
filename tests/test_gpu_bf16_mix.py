"""GPU parity of the bf16-mix edgewise path against a bf16-emulating oracle.

In the bf16 mode the only deliberate roundings are the two tensor-core operands: the
rotated, s^l_in-scaled input rows (A) and the radial table (B) are rounded to bf16,
everything else is float32.  The oracle applies exactly those two roundings to the
reference chain (bmm(f, P) -> block-diagonal mix -> bmm(., Q^T), float64 otherwise), so
the GPU result must match it to float32 accuracy (1e-4 relative L2) -- much tighter than
the 2e-2 bf16-mix bar, which could not tell a wrong interpolation weight from rounding.

Covers small and large representations, ragged tiles, a single edge, duplicate degrees,
log bins and a Cout that is not a multiple of 8.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import ops

pytestmark = pytest.mark.gpu

CASES = [
    # lvals_in, lvals_out, mult, E, log_bins
    ([0, 1, 2], [0, 1, 2], 64, 20000, False),        # config-3 shapes
    ([0, 1], [0, 1, 2, 3], 32, 5000, True),          # log bins, output blocks without input
    ([0, 1, 2], [0, 1], 16, 130, False),             # ragged tiles
    ([0, 1, 2], [0, 1, 2], 64, 1, False),            # a single edge
    ([0, 0, 1, 2], [0, 1, 1, 2], 32, 3000, False),   # duplicate degrees
    ([1, 2], [0, 2], 24, 999, False),                # three channel chunks, no l = 0 input
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 64, 3000, False),   # config-2 shapes
    ([2, 0, 1, 1], [1, 0], 7, 777, False),                 # Cout not a multiple of 8
]


def _lpos(lvals):
    lstd = np.concatenate([[l] * (2 * l + 1) for l in lvals])
    return torch.from_numpy(lstd[orc.m_first_perm(lvals)]).double()


def _bf16_oracle(f, dirs, dist, table, lin, lout, sh, p1, p2, nb, log):
    P, Q = orc.wigner_basis(dirs, lin).double(), orc.wigner_basis(dirs, lout).double()
    f_diag = torch.bmm(f.double(), P)
    d = dist.double()
    s = d / (d + sh)
    scale = s[:, None] ** _lpos(lin)[None, :]                     # s^l_in per m-first position
    a = (f_diag * scale[:, None, :]).float().to(torch.bfloat16).double() / scale[:, None, :]
    tb = table.float().to(torch.bfloat16).double()
    out = orc.block_diagonal_fwd(a, tb, d, lin, lout, sh, p1, p2, nb, log)
    return torch.bmm(out, Q.mT)


def _inputs(case, seed):
    lin, lout, mult, E, log = case
    torch.manual_seed(seed)
    rin, rout = fe.Repr(lin, mult=mult), fe.Repr(lout, mult=mult)
    layer = fe.EquivariantEdgewiseLinear(rin, rout, min_dist=0.5 if log else 0.0, log_bins=log)
    g = torch.Generator().manual_seed(seed + 1)
    f = torch.randn(E, mult, rin.dim(), generator=g)
    dirs = torch.randn(E, 3, generator=g)
    dist = torch.rand(E, generator=g) * 11 + 0.05          # beyond max_dist too (t > 1)
    if log:
        dist = dist.clamp(min=0.3)
    rw = layer.radial_weights
    with torch.no_grad():
        table = rw()
    p1, p2 = rw.binning_params()
    return layer, f, dirs, dist, table, p1, p2, rw.num_bins


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{c[1]}-C{c[2]}-E{c[3]}" for c in CASES])
def test_bf16_mix_matches_bf16_emulating_oracle(cuda_device, case):
    lin, lout, mult, E, log = case
    layer, f, dirs, dist, table, p1, p2, nb = _inputs(case, seed=4)
    dev = cuda_device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    y = ops.edgewise_fwd(f.to(dev), dist.to(dev), table.to(dev), lin, lout, mult, 0.1, p1, p2, nb, log,
                         directions=dirs.to(dev), status=status, mix="bf16")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = _bf16_oracle(f, dirs, dist, table, lin, lout, 0.1, p1, p2, nb, log)
    assert torch.isfinite(y).all()
    assert rel_l2(y, ref) < 1e-4
    # and within the bf16-mix bar of the unrounded reference
    exact = orc.edgewise_fwd(orc.wigner_basis(dirs, lin).double(), orc.wigner_basis(dirs, lout).double(),
                             f.double(), dist.double(), table.double(), lin, lout, 0.1, p1, p2, nb, log)
    assert rel_l2(y, exact) < 2e-2


def test_bf16_mix_deterministic_through_layer_and_gather(cuda_device):
    """The layer API (directions from LazyBasis) and the gathered form (x[src] inside the
    kernel, as the attention layer calls it) give the same bits, run after run."""
    dev = cuda_device
    r = fe.Repr([0, 1, 2], mult=64)
    layer = fe.EquivariantEdgewiseLinear(r, r).to(dev)
    layer.mix_precision = "bf16"
    g = torch.Generator().manual_seed(7)
    N, E = 3000, 40000
    x = torch.randn(N, 64, 9, generator=g).to(dev)
    src = torch.randint(0, N, (E,), generator=g).to(dev)
    dirs = torch.randn(E, 3, generator=g).to(dev)
    dist = (torch.rand(E, generator=g) * 10).to(dev)
    basis = fe.WignerDBasis([r])
    with torch.no_grad():
        P = basis.lazy(dirs)[0]
        a = layer(P, P, x[src], dist)
        b = layer(P, P, x[src], dist)
        c = layer._run(P, P, x, dist, src=src)
    assert torch.equal(a, b)
    assert torch.equal(a, c)
