"""The float64 backward restatement (oracle/block_diagonal_bwd_ref.c) against central finite
differences of the forward restatement (CPU only)."""
from __future__ import annotations

import pytest
import torch

import feq_oracle as orc


@pytest.mark.parametrize("lin,lout,log", [([0, 1, 2], [0, 1], False), ([1, 0, 2], [0, 2, 1], True)])
def test_backward_oracle_matches_finite_differences(lin, lout, log):
    g = torch.Generator().manual_seed(11)
    Cin, Cout, E, nb = 3, 2, 6, 8
    din, dout = sum(2 * l + 1 for l in lin), sum(2 * l + 1 for l in lout)
    W = orc.weight_dim(lin, lout)
    f = torch.randn(E, Cin, din, generator=g, dtype=torch.float64)
    tb = torch.randn(nb + 1, Cout, Cin, W, generator=g, dtype=torch.float64)
    d = torch.rand(E, generator=g, dtype=torch.float64) * 8.0 + 0.7
    go = torch.randn(E, Cout, dout, generator=g, dtype=torch.float64)
    p1, p2 = orc.binning_params(nb, 0.5, 10.0, log) if log else orc.binning_params(nb, 0.0, 10.0, False)
    gf, gt, gd = orc.block_diagonal_bwd(go, f, tb, d, lin, lout, 0.1, p1, p2, nb, log)
    loss = lambda f_, t_, d_: float((orc.block_diagonal_fwd(f_, t_, d_, lin, lout, 0.1, p1, p2, nb, log) * go).sum())
    eps = 1e-6
    for idx in [(0, 0, 0), (3, 1, din - 1), (5, 2, din // 2)]:
        a, b = f.clone(), f.clone()
        a[idx] += eps
        b[idx] -= eps
        assert abs((loss(a, tb, d) - loss(b, tb, d)) / (2 * eps) - float(gf[idx])) < 1e-6
    nz = torch.nonzero(gt)
    for r in nz[:: max(1, len(nz) // 4)][:4]:
        idx = tuple(int(x) for x in r)
        a, b = tb.clone(), tb.clone()
        a[idx] += eps
        b[idx] -= eps
        assert abs((loss(f, a, d) - loss(f, b, d)) / (2 * eps) - float(gt[idx])) < 1e-6
    for e in range(E):
        a, b = d.clone(), d.clone()
        a[e] += eps
        b[e] -= eps
        fd = (loss(f, tb, a) - loss(f, tb, b)) / (2 * eps)
        assert abs(fd - float(gd[e])) < 1e-5 * max(1.0, abs(fd))
