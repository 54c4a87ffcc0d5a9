"""GPU parity of the tensor-core (tcgen05) radial mix inside the fused edgewise op.

Modes and tolerances (relative L2 against the CPU oracle of the reference path):
  "bf16x3"  every operand split into two bf16 terms   -> 1e-4 (the fp32 bar)
  "bf16"    bf16 operands, fp32 accumulation          -> 2e-2 (the bf16-mix bar)
The status word must stay 0 (1 = bad src index, 2 = a tensor-core wait timed out).
"""
from __future__ import annotations

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import ops

pytestmark = pytest.mark.gpu

TOL = {"bf16x3": 1e-4, "bf16": 2e-2}

CASES = [
    # lvals_in, lvals_out, mult, E, log_bins
    ([0, 1, 2], [0, 1, 2], 64, 30000, False),                  # config-3 shapes
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 64, 6000, False),       # config-2 shapes
    ([0, 1, 2, 3], [0, 1, 2, 3], 128, 3000, False),            # config-4 hidden shapes
    ([0, 1], [0, 1, 2, 3], 32, 5000, True),                    # log bins, empty output blocks
    ([2, 0, 1, 1], [1, 0], 7, 777, False),                     # K and N padding, duplicates
    ([0, 1, 2], [0, 1, 2], 16, 1, False),                      # a single edge
    ([0, 1, 2], [0, 1], 16, 130, False),                       # ragged tiles
]


def _run(case, mode, dev, dense=False, seed=0):
    lin, lout, mult, E, log_bins = case
    torch.manual_seed(seed)
    rin, rout = fe.Repr(lin, mult=mult), fe.Repr(lout, mult=mult)
    layer = fe.EquivariantEdgewiseLinear(rin, rout, min_dist=0.5 if log_bins else 0.0, log_bins=log_bins).to(dev)
    g = torch.Generator().manual_seed(seed + 1)
    f = torch.randn(E, mult, rin.dim(), generator=g)
    dirs = torch.randn(E, 3, generator=g)
    dist = torch.rand(E, generator=g) * 11 - 0.5
    if log_bins:
        dist = dist.abs() + 0.3
    P, Q = fe.WignerDBasis([rin, rout])(dirs.to(dev))
    if dense:
        P, Q = P.clone(), Q.clone()
    rw = layer.radial_weights
    with torch.no_grad():
        table = rw()
    p1, p2 = rw.binning_params()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kw = dict(P=P, Q=Q) if dense else dict(directions=dirs.to(dev))
    y = ops.edgewise_fwd(f.to(dev), dist.to(dev), table, lin, lout, mult, 0.1, p1, p2, rw.num_bins, log_bins,
                         status=status, mix=mode, **kw)
    torch.cuda.synchronize()
    ref = orc.edgewise_fwd(orc.wigner_basis(dirs, lin), orc.wigner_basis(dirs, lout), f, dist, table.cpu(), lin,
                           lout, 0.1, p1, p2, rw.num_bins, log_bins)
    return y, ref, int(status.item())


@pytest.mark.parametrize("mode", ["bf16x3", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{c[1]}-C{c[2]}-E{c[3]}" for c in CASES])
def test_tc_mix_matches_oracle(cuda_device, mode, case):
    y, ref, st = _run(case, mode, cuda_device)
    assert st == 0
    assert torch.isfinite(y).all()
    assert rel_l2(y, ref) < TOL[mode]


@pytest.mark.parametrize("mode", ["bf16x3"])
def test_tc_mix_dense_basis(cuda_device, mode):
    y, ref, st = _run(([0, 1, 2], [0, 1, 2, 3], 32, 4000, False), mode, cuda_device, dense=True)
    assert st == 0 and rel_l2(y, ref) < TOL[mode]


def test_tc_mix_deterministic_and_layer_attribute(cuda_device):
    r = fe.Repr([0, 1, 2], mult=64)
    layer = fe.EquivariantEdgewiseLinear(r, r).to(cuda_device)
    g = torch.Generator().manual_seed(3)
    f = torch.randn(20000, 64, 9, generator=g).to(cuda_device)
    dirs = torch.randn(20000, 3, generator=g).to(cuda_device)
    dist = (torch.rand(20000, generator=g) * 10).to(cuda_device)
    P, Q = fe.WignerDBasis([r, r])(dirs)
    with torch.no_grad():
        y32 = layer(P, Q, f, dist)
        layer.mix_precision = "bf16x3"
        a = layer(P, Q, f, dist)
        b = layer(P, Q, f, dist)
    assert torch.equal(a, b)
    assert rel_l2(a, y32) < 1e-4
