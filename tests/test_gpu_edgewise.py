"""GPU parity of the fused edgewise linear and of block_diagonal_cuda.

Tolerance: relative L2 <= 1e-4 against the oracle / reference fixtures (the
fp32 bar of the tier); equivariance max-relative 1e-4 as the reference's
tests/test_equivariance.py:96-99.
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import ROOT, check_equivariance, golden, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _layer_from_case(case, dev):
    rin = fe.Repr(case["lvals_in"], mult=case["mult_in"])
    rout = fe.Repr(case["lvals_out"], mult=case["mult_out"])
    layer = fe.EquivariantEdgewiseLinear(rin, rout, num_bins=case["num_bins"], min_dist=case["min_dist"],
                                         max_dist=case["max_dist"], log_bins=case["log_bins"])
    layer.load_state_dict(case["state"])
    return layer.to(dev), rin, rout


@pytest.mark.parametrize("idx", range(17))
def test_edgewise_matches_reference_fixture(cuda_device, idx):
    case = golden("edgewise.pt")[idx]
    layer, rin, rout = _layer_from_case(case, cuda_device)
    P, Q = fe.WignerDBasis([rin, rout])(case["directions"].to(cuda_device))
    with torch.no_grad():
        y = layer(P, Q, case["features"].to(cuda_device), case["distances"].to(cuda_device))
        y_dense = layer(P.clone(), Q.clone(), case["features"].to(cuda_device), case["distances"].to(cuda_device))
    assert rel_l2(y, case["output"]) < TOL
    assert rel_l2(y_dense, case["output"]) < TOL        # dense-P path (arbitrary matrices)


def test_edgewise_cfg1_small(cuda_device):
    fx = golden("edgewise_cfg1_small.pt")
    rr = fe.Repr([0, 1, 2], mult=32)
    layer = fe.EquivariantEdgewiseLinear(rr, rr, num_bins=100, min_dist=0.0, max_dist=10.0)
    layer.load_state_dict(fx["state"])
    layer = layer.to(cuda_device)
    coords, src, dst = fx["coords"].to(cuda_device), fx["src"].to(cuda_device), fx["dst"].to(cuda_device)
    vec = coords[dst] - coords[src]
    P, Q = fe.WignerDBasis([rr, rr])(vec)
    x = fx["x"].to(cuda_device)
    with torch.no_grad():
        y = layer(P, Q, x[src], vec.norm(dim=-1))
        y_gather = layer._run(P, Q, x, vec.norm(dim=-1), src=src)       # fused gather
    assert rel_l2(y, fx["output"]) < TOL
    assert torch.equal(y, y_gather)


def _oracle_layer_output(layer, P, Q, f, dist, lin, lout):
    rw = layer.radial_weights
    with torch.no_grad():
        table = rw().cpu()
    p1, p2 = rw.binning_params()
    return orc.edgewise_fwd(P.cpu(), Q.cpu(), f.cpu(), dist.cpu(), table, lin, lout,
                            layer.solid_harmonic_scale, p1, p2, rw.num_bins, rw.log)


@pytest.mark.parametrize("lin,lout,mult,E", [
    ([0, 1, 2], [0, 1, 2], 64, 30000),       # config-3 shapes
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 64, 6000),   # config-2 shapes
    ([0, 1, 2, 3], [0, 1, 2, 3], 128, 3000),   # config-4 hidden shapes (ci chunking)
    ([0, 1], [0, 1, 2, 3], 32, 5000),
    ([2, 0, 1, 1], [1, 0], 7, 777),
    ([0, 1, 2, 3, 4, 5, 6], [0, 2, 4, 6], 8, 500),
])
def test_edgewise_matches_oracle_large(cuda_device, lin, lout, mult, E):
    torch.manual_seed(0)
    rin, rout = fe.Repr(lin, mult=mult), fe.Repr(lout, mult=mult)
    layer = fe.EquivariantEdgewiseLinear(rin, rout).to(cuda_device)
    g = torch.Generator().manual_seed(1)
    f = torch.randn(E, mult, rin.dim(), generator=g)
    dirs = torch.randn(E, 3, generator=g)
    dist = torch.rand(E, generator=g) * 11 - 0.5      # includes extrapolation both sides
    P, Q = fe.WignerDBasis([rin, rout])(dirs.to(cuda_device))
    with torch.no_grad():
        y = layer(P, Q, f.to(cuda_device), dist.to(cuda_device))
    ref = _oracle_layer_output(layer, P, Q, f, dist, lin, lout)
    assert rel_l2(y, ref) < TOL


LVALS_CONFIGS = [([0], [0]), ([1], [1]), ([2], [2]), ([0, 1], [0, 1]), ([0, 1, 2], [0, 1, 2]),
                 ([1, 2], [1, 2]), ([0, 2], [0, 2]), ([1, 2, 3], [1, 2, 3]), ([0], [0, 1]),
                 ([0, 1], [0, 1, 2]), ([1], [0, 1]), ([1, 2], [0, 1, 2]), ([0, 1, 2], [1, 2]),
                 ([2], [0, 1, 2]), ([0, 1], [2]), ([0, 0], [0, 0]), ([1, 1], [1, 1]),
                 ([0, 1, 1], [0, 1, 1]), ([1, 2, 2], [1, 2, 2]), ([0, 1, 1], [0, 1, 2]), ([1, 2, 2], [0, 1])]


@pytest.mark.parametrize("lin,lout", LVALS_CONFIGS)
def test_equivariance(cuda_device, lin, lout):
    """tests/test_equivariance.py:47-99 of the reference, on the B200 path."""
    torch.manual_seed(42)
    mult, N, E = 4, 20, 50
    rin, rout = fe.Repr(lin, mult=mult), fe.Repr(lout, mult=mult)
    layer = fe.EquivariantEdgewiseLinear(rin, rout, num_bins=50).to(cuda_device)
    basis = fe.WignerDBasis([rin, rout]).to(cuda_device)
    x = torch.randn(N, mult, rin.dim(), device=cuda_device)
    src = torch.randint(0, N, (E,), device=cuda_device)
    dist = torch.rand(E, device=cuda_device) * 5.0
    dirs = torch.randn(E, 3, device=cuda_device)
    dirs = dirs / dirs.norm(dim=-1, keepdim=True)
    axis, angle = fe.random_rotation(device=cuda_device)
    D_in = fe.WignerD(rin).to(cuda_device).rot(axis, angle)
    D_out = fe.WignerD(rout).to(cuda_device).rot(axis, angle)
    R = fe.WignerD(fe.Repr([1])).to(cuda_device).rot(axis, angle, cartesian=True)
    with torch.no_grad():
        P, Q = basis(dirs)
        y1 = torch.einsum("ij,ecj->eci", D_out, layer(P, Q, x[src], dist))
        xr = torch.einsum("ij,ncj->nci", D_in, x)
        P2, Q2 = basis(torch.einsum("ij,ej->ei", R, dirs))
        y2 = layer(P2, Q2, xr[src], dist)
    assert y1.abs().mean().item() > 0.01
    check_equivariance(y1, y2, rtol=1e-4)


def test_self_loop_suppresses_higher_l(cuda_device):
    r = fe.Repr([0, 1, 2], mult=8)
    layer = fe.EquivariantEdgewiseLinear(r, r).to(cuda_device)
    P, Q = fe.WignerDBasis([r, r])(torch.zeros(10, 3, device=cuda_device))
    with torch.no_grad():
        y = layer(P, Q, torch.randn(10, 8, 9, device=cuda_device), torch.zeros(10, device=cuda_device))
    assert torch.isfinite(y).all()
    assert y[..., 1:].abs().max() < 1e-6 and y[..., 0].abs().max() > 0


def test_edge_cases(cuda_device):
    r = fe.Repr([0, 1, 2], mult=4)
    layer = fe.EquivariantEdgewiseLinear(r, r).to(cuda_device)
    basis = fe.WignerDBasis([r, r])
    with torch.no_grad():
        P, Q = basis(torch.randn(0, 3, device=cuda_device))
        assert layer(P, Q, torch.randn(0, 4, 9, device=cuda_device), torch.rand(0, device=cuda_device)).shape == (0, 4, 9)
        P, Q = basis(torch.randn(1, 3, device=cuda_device))
        y = layer(P, Q, torch.randn(1, 4, 9, device=cuda_device), torch.rand(1, device=cuda_device))
        assert y.shape == (1, 4, 9) and torch.isfinite(y).all()
        P, Q = basis(torch.randn(4, 3, device=cuda_device))
        d = torch.tensor([-5.0, 0.0, 5.0, 100.0], device=cuda_device)
        assert torch.isfinite(layer(P, Q, torch.randn(4, 4, 9, device=cuda_device), d)).all()


def test_deterministic(cuda_device):
    r = fe.Repr([0, 1, 2, 3], mult=16)
    layer = fe.EquivariantEdgewiseLinear(r, r).to(cuda_device)
    g = torch.Generator().manual_seed(9)
    f = torch.randn(20000, 16, 16, generator=g).to(cuda_device)
    dirs = torch.randn(20000, 3, generator=g).to(cuda_device)
    dist = (torch.rand(20000, generator=g) * 10).to(cuda_device)
    P, Q = fe.WignerDBasis([r, r])(dirs)
    with torch.no_grad():
        a = layer(P, Q, f, dist)
        b = layer(P, Q, f, dist)
    assert torch.equal(a, b)


@pytest.mark.parametrize("gather", [False, True])
def test_edge_range_chunking_is_exact(cuda_device, gather, monkeypatch):
    """A call whose scratch exceeds the cap runs as consecutive edge ranges: the result is
    bit-identical to the single call (edges are independent)."""
    from flash_eq.cuda import ops

    r = fe.Repr([0, 1, 2], mult=32)
    layer = fe.EquivariantEdgewiseLinear(r, r).to(cuda_device)
    g = torch.Generator().manual_seed(12)
    E, N = 7001, 900
    dirs = torch.randn(E, 3, generator=g).to(cuda_device)
    dist = (torch.rand(E, generator=g) * 10).to(cuda_device)
    if gather:
        x = torch.randn(N, 32, 9, generator=g).to(cuda_device)
        src = torch.randint(0, N, (E,), generator=g).to(cuda_device)
        ea = torch.randn(E, 32, 9, generator=g).to(cuda_device)
        bases = fe.WignerDBasis([r, r]).lazy(dirs)
        call = lambda: layer._run(bases[0], bases[1], x, dist, src=src, edge_add=ea)
    else:
        f = torch.randn(E, 32, 9, generator=g).to(cuda_device)
        P, Q = fe.WignerDBasis([r, r])(dirs)
        call = lambda: layer(P, Q, f, dist)
    with torch.no_grad():
        whole = call()
        monkeypatch.setattr(ops, "EDGEWISE_WS_CAP", 1 << 20)
        parts = call()
    assert torch.equal(whole, parts)


@pytest.mark.parametrize("lin,lout,mult,E,log_bins", [
    ([0, 1, 2], [0, 1, 2], 32, 5000, False), ([0, 1, 2, 3, 4], [0, 1], 16, 2000, True),
    ([1, 2, 2], [0, 1], 5, 333, False), ([0], [0, 1, 2], 3, 1, False)])
def test_block_diagonal_cuda_matches_oracle(cuda_device, lin, lout, mult, E, log_bins):
    from flash_eq.cuda import block_diagonal_cuda
    g = torch.Generator().manual_seed(4)
    rin, rout = fe.Repr(lin, mult), fe.Repr(lout, mult)
    pr = fe.ProductRepr(rin, rout)
    nb = 64
    table = torch.randn(nb + 1, mult, mult, pr.nreps(), generator=g)
    f = torch.randn(E, mult, rin.dim(), generator=g)
    dist = torch.rand(E, generator=g) * 12 - 1
    p1, p2 = orc.binning_params(nb, 0.5 if log_bins else 0.0, 10.0, log_bins)
    ref = orc.block_diagonal_fwd(f, table, dist, lin, lout, 0.1, p1, p2, nb, log_bins)
    y = block_diagonal_cuda(f.to(cuda_device), table.to(cuda_device), dist.to(cuda_device), pr, p1, p2, nb,
                            log_bins, 0.1)
    assert rel_l2(y, ref) < TOL


def _reference_kernel():
    hits = glob.glob(os.path.join(ROOT, "oracle", "_ref", "_block_diagonal_cuda*.so"))
    if not hits:
        return None
    loader = importlib.machinery.ExtensionFileLoader("_block_diagonal_cuda", hits[0])
    spec = importlib.util.spec_from_file_location("_block_diagonal_cuda", hits[0], loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


REF_KERNEL_CASES = [
    # lvals_in, lvals_out, mult, E, num_bins, log_bins, mix, tolerance
    ([0, 1, 2], [0, 1, 2], 16, 3000, 50, False, "fp32", 1e-5),
    ([0, 1, 1, 3], [2, 0], 6, 999, 50, False, "fp32", 1e-5),
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 64, 4000, 100, False, "fp32", 1e-5),     # config-2 shapes
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 64, 4000, 100, False, "bf16x3", 1e-4),
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 64, 4000, 100, False, "bf16", 2e-2),
    ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4], 64, 3000, 100, True, "bf16x3", 1e-4),     # log bins
    ([0, 1, 2], [0, 1, 2], 64, 6000, 100, True, "fp32", 1e-5),
    ([0, 1], [0, 1, 2, 3], 32, 2000, 64, False, "bf16x3", 1e-4),
]


@pytest.mark.parametrize("case", REF_KERNEL_CASES, ids=lambda c: f"L{max(c[0])}-{max(c[1])}_C{c[2]}_"
                         f"{'log' if c[5] else 'lin'}_{c[6]}")
def test_block_diagonal_matches_reference_cuda_kernel(cuda_device, case):
    """Second oracle: the reference's own kernel compiled for sm_100a (oracle/_ref), at small
    shapes and at the benched config-2 shapes (L <= 4, mult 64), linear and log bins, for the
    CUDA-core (fp32) mix and both tensor-core mixes."""
    ref = _reference_kernel()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    from flash_eq.cuda import block_diagonal_cuda
    lin, lout, mult, E, nb, log_bins, mix, tol = case
    g = torch.Generator().manual_seed(5 + E)
    rin, rout = fe.Repr(lin, mult), fe.Repr(lout, mult)
    pr = fe.ProductRepr(rin, rout)
    table = torch.randn(nb + 1, mult, mult, pr.nreps(), generator=g).to(cuda_device)
    f = torch.randn(E, mult, rin.dim(), generator=g).to(cuda_device)
    if log_bins:
        lo_d, hi_d = 0.5, 10.0
        dist = (lo_d + torch.rand(E, generator=g) * (hi_d - lo_d)).to(cuda_device)
        p1, p2 = orc.binning_params(nb, lo_d, hi_d, True)
    else:
        dist = (torch.rand(E, generator=g) * 10).to(cuda_device)
        p1, p2 = 0.0, nb / 10.0
    lvi = torch.tensor(lin, dtype=torch.int32, device=cuda_device)
    lvo = torch.tensor(lout, dtype=torch.int32, device=cuda_device)
    mi = max(max(lin), max(lout))
    max_in = max((1 if m == 0 else 2) * sum(l >= m for l in lin) for m in range(mi + 1))
    (yr,) = ref.forward(f, table, dist, 0.1, p1, p2, nb, log_bins, lvi, lvo, mult, rout.dim(), max_in)
    y = block_diagonal_cuda(f, table, dist, pr, p1, p2, nb, log_bins, 0.1, mix=mix)
    assert rel_l2(y, yr) < tol
