"""GPU parity of the one-kernel separable edgewise linear (feq_edgewise_separable_fwd).

The kernel never forms the radial table: it interpolates the radial net's features per
edge and applies the channel patterns on the tensor cores.  It must give the result of
the reference formulation -- table = einsum(channel_patterns, features), then
bmm(f, P) -> block_diagonal_cuda -> bmm(., Q^T) (flash_eq/layers/linear.py:100-160) --
computed here by the CPU oracle from the same table.

Tolerances (relative L2): 1e-4 for bf16x3 (the float32 bar), 2e-2 for bf16.
"""
from __future__ import annotations

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import _lib, ops

pytestmark = pytest.mark.gpu

TOL = {"bf16x3": 1e-4, "bf16": 2e-2}

CASES = [
    # L, E, gather, edge_add, log_bins
    (2, 30000, False, False, False),
    (4, 6000, False, False, False),
    (1, 5003, True, False, False),
    (3, 4097, True, True, False),
    (2, 7777, True, True, True),
    (4, 1, False, False, False),
    (2, 3, True, False, False),
    (4, 130, True, False, True),
]


def _case(dev, L, E, gather, edge_add, log_bins, seed=0):
    torch.manual_seed(seed)
    r = fe.Repr(list(range(L + 1)), mult=64)
    layer = fe.EquivariantEdgewiseLinear(r, r, min_dist=0.5 if log_bins else 0.0, log_bins=log_bins).to(dev).eval()
    g = torch.Generator().manual_seed(seed + 11)
    n_rows = max(1, E // 3) if gather else E
    x = torch.randn(n_rows, 64, r.dim(), generator=g)
    src = torch.randint(0, n_rows, (E,), generator=g) if gather else None
    ea = torch.randn(E, 64, r.dim(), generator=g) if edge_add else None
    dirs = torch.randn(E, 3, generator=g)
    dist = torch.rand(E, generator=g) * 11 - 0.5
    if log_bins:
        dist = dist.abs() + 0.3
    return layer, r, x, src, ea, dirs, dist


def _oracle(layer, lv, x, src, ea, dirs, dist):
    rw = layer.radial_weights
    with torch.no_grad():
        table = rw().cpu()
    p1, p2 = rw.binning_params()
    f = x[src] if src is not None else x
    if ea is not None:
        f = f + ea
    P = orc.wigner_basis(dirs, lv)
    return orc.edgewise_fwd(P, P, f, dist, table, lv, lv, layer.solid_harmonic_scale, p1, p2, rw.num_bins,
                            rw.log)


@pytest.mark.parametrize("mix", ["bf16x3", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"L{c[0]}_E{c[1]}{'_src' if c[2] else ''}"
                         f"{'_add' if c[3] else ''}{'_log' if c[4] else ''}")
def test_separable_matches_oracle(cuda_device, case, mix):
    L, E, gather, edge_add, log_bins = case
    layer, r, x, src, ea, dirs, dist = _case(cuda_device, *case)
    lv = list(range(L + 1))
    rw = layer.radial_weights
    assert ops.separable_supported(lv, lv, 64, 64, rw.rank, mix)
    p1, p2 = rw.binning_params()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    with torch.no_grad():
        y = ops.edgewise_separable_fwd(
            x.to(cuda_device), dist.to(cuda_device), rw.channel_patterns, rw.radial_features(), lv, lv,
            layer.solid_harmonic_scale, p1, p2, rw.num_bins, rw.log, directions=dirs.to(cuda_device),
            src=None if src is None else src.to(cuda_device), edge_add=None if ea is None else ea.to(cuda_device),
            status=status, mix=mix)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = _oracle(layer, lv, x, src, ea, dirs, dist)
    assert torch.isfinite(y).all()
    assert rel_l2(y, ref) < TOL[mix]


@pytest.mark.parametrize("mix", ["bf16x3", "bf16"])
def test_layer_routes_through_the_separable_kernel(cuda_device, mix):
    """EquivariantEdgewiseLinear under no_grad with a WignerDBasis basis takes the one-kernel
    path (two library launches: the radial net's features, then the edgewise kernel) and
    agrees with the oracle."""
    layer, r, x, src, ea, dirs, dist = _case(cuda_device, 2, 20000, False, False, False, seed=4)
    layer.mix_precision = mix
    lib = _lib.load()
    P, Q = fe.WignerDBasis([r, r])(dirs.to(cuda_device))
    n0 = lib.feq_launch_count()
    with torch.no_grad():
        y = layer(P, Q, x.to(cuda_device), dist.to(cuda_device))
    torch.cuda.synchronize()
    assert lib.feq_launch_count() - n0 == 2
    ref = _oracle(layer, [0, 1, 2], x, src, ea, dirs, dist)
    assert rel_l2(y, ref) < TOL[mix]


def test_separable_is_deterministic(cuda_device):
    layer, r, x, src, ea, dirs, dist = _case(cuda_device, 4, 9000, True, False, False, seed=7)
    rw = layer.radial_weights
    p1, p2 = rw.binning_params()
    lv = [0, 1, 2, 3, 4]
    args = [x.to(cuda_device), dist.to(cuda_device), rw.channel_patterns, rw.radial_features().detach(), lv, lv,
            0.1, p1, p2, rw.num_bins, False]
    kw = dict(directions=dirs.to(cuda_device), src=src.to(cuda_device))
    with torch.no_grad():
        a = ops.edgewise_separable_fwd(*args, **kw)
        b = ops.edgewise_separable_fwd(*args, **kw)
    assert torch.equal(a, b)


def test_separable_bad_src_sets_status_1(cuda_device):
    layer, r, x, src, ea, dirs, dist = _case(cuda_device, 2, 500, True, False, False, seed=9)
    src = src.clone()
    src[17] = x.shape[0] + 5
    src[301] = -1
    rw = layer.radial_weights
    p1, p2 = rw.binning_params()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    with torch.no_grad():
        y = ops.edgewise_separable_fwd(x.to(cuda_device), dist.to(cuda_device), rw.channel_patterns,
                                       rw.radial_features(), [0, 1, 2], [0, 1, 2], 0.1, p1, p2, rw.num_bins, False,
                                       directions=dirs.to(cuda_device), src=src.to(cuda_device), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert torch.count_nonzero(y[17]) == 0 and torch.count_nonzero(y[301]) == 0   # bad rows read as zero
    assert torch.isfinite(y).all()


@pytest.mark.parametrize("L", [1, 2, 4])
def test_separable_equivariance(cuda_device, L):
    """tests/test_equivariance.py:47-99 of the reference, through the layer at mult 64 (the
    shapes the one-kernel path serves): rotating the inputs and the directions by R rotates
    the output by R."""
    from conftest import check_equivariance
    torch.manual_seed(42)
    r = fe.Repr(list(range(L + 1)), mult=64)
    layer = fe.EquivariantEdgewiseLinear(r, r, num_bins=50).to(cuda_device).eval()
    basis = fe.WignerDBasis([r, r]).to(cuda_device)
    N, E = 40, 300
    x = torch.randn(N, 64, r.dim(), device=cuda_device)
    src = torch.randint(0, N, (E,), device=cuda_device)
    dist = torch.rand(E, device=cuda_device) * 5.0
    dirs = torch.randn(E, 3, device=cuda_device)
    dirs = dirs / dirs.norm(dim=-1, keepdim=True)
    axis, angle = fe.random_rotation(device=cuda_device)
    D = fe.WignerD(r).to(cuda_device).rot(axis, angle)
    R = fe.WignerD(fe.Repr([1])).to(cuda_device).rot(axis, angle, cartesian=True)
    with torch.no_grad():
        P, Q = basis(dirs)
        y1 = torch.einsum("ij,ecj->eci", D, layer(P, Q, x[src], dist))
        xr = torch.einsum("ij,ncj->nci", D, x)
        P2, Q2 = basis(torch.einsum("ij,ej->ei", R, dirs))
        y2 = layer(P2, Q2, xr[src], dist)
    assert y1.abs().mean().item() > 0.01
    check_equivariance(y1, y2, rtol=1e-4)
