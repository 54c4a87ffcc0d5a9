"""GPU parity of the block-diagonal backward (grad_features, grad_table, grad_distances)
against the float64 CPU restatement of the reference backward kernels, plus the autograd
wrapper and determinism.  Tolerances (relative L2): bf16x3 1e-4, bf16 2e-2."""
from __future__ import annotations

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import block_diagonal_cuda, ops

pytestmark = pytest.mark.gpu

TOL = {"bf16x3": 1e-4, "bf16": 2e-2}

CASES = [
    # lvals_in, lvals_out, Cin, Cout, E, log_bins
    ([0, 1, 2], [0, 1, 2], 16, 16, 3000, False),
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 8, 8, 700, False),
    ([0, 1], [0, 1, 2, 3], 12, 20, 900, True),
    ([2, 0, 1, 1], [1, 0], 7, 5, 333, False),
    ([0, 1, 2], [0, 1], 64, 64, 1200, False),
    ([0, 1, 2], [0, 1, 2], 4, 4, 1, False),
]


def _inputs(case, seed=0):
    lin, lout, cin, cout, E, log = case
    g = torch.Generator().manual_seed(seed)
    din, dout = sum(2 * l + 1 for l in lin), sum(2 * l + 1 for l in lout)
    W = orc.weight_dim(lin, lout)
    nb = 50
    f = torch.randn(E, cin, din, generator=g)
    tb = torch.randn(nb + 1, cout, cin, W, generator=g) * 0.3
    if log:
        d = torch.rand(E, generator=g) * 9.0 + 0.6
        p1, p2 = orc.binning_params(nb, 0.5, 10.0, True)
    else:
        d = torch.rand(E, generator=g) * 11.0 + 0.05       # includes distances beyond max (t > 1)
        p1, p2 = orc.binning_params(nb, 0.0, 10.0, False)
    go = torch.randn(E, cout, dout, generator=g)
    return lin, lout, f, tb, d, go, p1, p2, nb, log


@pytest.mark.parametrize("mode", ["bf16x3", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{c[1]}-{c[2]}x{c[3]}-E{c[4]}" for c in CASES])
def test_backward_matches_oracle(cuda_device, mode, case):
    lin, lout, f, tb, d, go, p1, p2, nb, log = _inputs(case)
    gf, gt, gd = ops.block_diagonal_bwd(go.to(cuda_device), f.to(cuda_device), tb.to(cuda_device),
                                        d.to(cuda_device), lin, lout, 0.1, p1, p2, nb, log, mix=mode)
    torch.cuda.synchronize()
    rf, rt, rd = orc.block_diagonal_bwd(go, f, tb, d, lin, lout, 0.1, p1, p2, nb, log)
    assert rel_l2(gf, rf) < TOL[mode]
    assert rel_l2(gt, rt) < TOL[mode]
    assert rel_l2(gd, rd) < TOL[mode]


def test_backward_deterministic_and_autograd(cuda_device):
    lin, lout, f, tb, d, go, p1, p2, nb, log = _inputs(CASES[0], seed=3)
    dev = cuda_device
    a = ops.block_diagonal_bwd(go.to(dev), f.to(dev), tb.to(dev), d.to(dev), lin, lout, 0.1, p1, p2, nb, log)
    b = ops.block_diagonal_bwd(go.to(dev), f.to(dev), tb.to(dev), d.to(dev), lin, lout, 0.1, p1, p2, nb, log)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    pr = fe.ProductRepr(fe.Repr(lin, 1), fe.Repr(lout, 1))
    fx = f.to(dev).requires_grad_()
    tx = tb.to(dev).requires_grad_()
    dx = d.to(dev).requires_grad_()
    out = block_diagonal_cuda(fx, tx, dx, pr, p1, p2, nb, log, 0.1)
    out.backward(go.to(dev))
    rf, rt, rd = orc.block_diagonal_bwd(go, f, tb, d, lin, lout, 0.1, p1, p2, nb, log)
    assert rel_l2(fx.grad, rf) < 1e-4 and rel_l2(tx.grad, rt) < 1e-4 and rel_l2(dx.grad, rd) < 1e-4


def test_backward_zero_distance_nan_like_reference(cuda_device):
    lin, lout, f, tb, d, go, p1, p2, nb, log = _inputs(([0, 1], [0, 1], 4, 4, 64, False), seed=5)
    d[::7] = 0.0
    gf, gt, gd = ops.block_diagonal_bwd(go.to(cuda_device), f.to(cuda_device), tb.to(cuda_device),
                                        d.to(cuda_device), lin, lout, 0.1, p1, p2, nb, log)
    rf, rt, rd = orc.block_diagonal_bwd(go, f, tb, d, lin, lout, 0.1, p1, p2, nb, log)
    assert torch.equal(torch.isnan(gd.cpu()), torch.isnan(rd))
    ok = ~torch.isnan(rd)
    assert rel_l2(gd.cpu()[ok], rd[ok]) < 1e-4
    assert rel_l2(gf, rf) < 1e-4 and rel_l2(gt, rt) < 1e-4


def test_edgewise_layer_training_step_matches_oracle(cuda_device):
    """Gradients of EquivariantEdgewiseLinear (inputs and radial-MLP parameters) against the
    oracle chain bmm -> block-diagonal backward -> bmm, with the table's own autograd."""
    dev = cuda_device
    lin, lout = [0, 1, 2], [0, 1]
    torch.manual_seed(0)
    rin, rout = fe.Repr(lin, mult=8), fe.Repr(lout, mult=6)
    layer = fe.EquivariantEdgewiseLinear(rin, rout).to(dev)
    ref_layer = fe.EquivariantEdgewiseLinear(rin, rout).to(dev)
    ref_layer.load_state_dict(layer.state_dict())
    g = torch.Generator().manual_seed(2)
    E = 500
    x = torch.randn(E, 8, rin.dim(), generator=g)
    dirs = torch.randn(E, 3, generator=g)
    dist = torch.rand(E, generator=g) * 9 + 0.2
    go = torch.randn(E, 6, rout.dim(), generator=g)
    P, Q = fe.WignerDBasis([rin, rout])(dirs.to(dev))
    xg = x.to(dev).requires_grad_()
    out = layer(P, Q, xg, dist.to(dev))
    out.backward(go.to(dev))
    # oracle chain on the same table
    rw = ref_layer.radial_weights
    table = rw()
    p1, p2 = rw.binning_params()
    Pc, Qc = P.double().cpu(), Q.double().cpu()
    f_diag = torch.bmm(x.double(), Pc)
    go_diag = torch.bmm(go.double(), Qc)                      # d/d out_diag of <go, out_diag Q^T>
    gfd, gtab, _ = orc.block_diagonal_bwd(go_diag, f_diag, table.detach().double().cpu(), dist.double(), lin, lout,
                                          layer.solid_harmonic_scale, p1, p2, rw.num_bins, rw.log)
    gx = torch.bmm(gfd, Pc.mT)
    assert rel_l2(xg.grad, gx) < 1e-4
    table.backward(gtab.to(dev, torch.float32))
    for (n, a), (_, b) in zip(layer.named_parameters(), ref_layer.named_parameters()):
        assert rel_l2(a.grad, b.grad) < 1e-4, n


@pytest.mark.parametrize("mode", ["bf16x3", "bf16"])
@pytest.mark.parametrize("case", CASES[:5], ids=[f"{c[0]}-{c[1]}" for c in CASES[:5]])
def test_block_diagonal_tensor_core_forward(cuda_device, mode, case):
    lin, lout, f, tb, d, go, p1, p2, nb, log = _inputs(case, seed=9)
    y = ops.block_diagonal_fwd(f.to(cuda_device), tb.to(cuda_device), d.to(cuda_device), lin, lout, 0.1, p1, p2, nb,
                               log, mix=mode)
    ref = orc.block_diagonal_fwd(f.double(), tb.double(), d.double(), lin, lout, 0.1, p1, p2, nb, log)
    assert rel_l2(y, ref) < TOL[mode]
