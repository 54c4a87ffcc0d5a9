"""GPU parity: Wigner-D basis, distance binning, edge sort (CUDA path vs oracle).

Tolerances: basis entries 2e-5 absolute against the reference's float32
matrix_exp (both are float32; the closed form itself is exact to 1e-9, see
test_abi_and_host.py); bin indices and sort permutation/offsets bit-exact.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import golden
from flash_eq.cuda import ops

pytestmark = pytest.mark.gpu


def test_basis_matches_reference_fixture(cuda_device):
    fx = golden("basis.pt")
    dirs = fx["directions"].to(cuda_device)
    for key, P in fx.items():
        if not key.startswith("P_"):
            continue
        lv = [int(x) for x in key[2:].split(",")]
        (ours,) = fe.WignerDBasis([fe.Repr(lv)])(dirs)
        err = (ours.cpu() - P).abs().max().item()
        assert err < 2e-5, (key, err)
        assert torch.isfinite(ours).all()


def test_rot_to_ez_matches_reference_fixture(cuda_device):
    fx = golden("basis.pt")
    ours = fe.WignerD(fe.Repr([0, 1, 2])).to(cuda_device).rot_to_ez(fx["directions"].to(cuda_device))
    assert (ours.cpu() - fx["rot_to_ez_0,1,2"]).abs().max().item() < 2e-5


@pytest.mark.parametrize("lvals", [[0, 1, 2, 3, 4], [0, 1, 1, 2], [3, 0, 2], [6], [0, 1, 2, 3, 4, 5, 6]])
def test_basis_matches_oracle_large(cuda_device, lvals):
    g = torch.Generator().manual_seed(7)
    dirs = torch.cat([torch.randn(4000, 3, generator=g), torch.randn(200, 3, generator=g) * 1e-6,
                      torch.tensor([[0.0, 0, 0], [0, 0, 1], [0, 0, -1], [1e-4, 0, -1], [0, 2e-7, 1]])])
    ref = orc.wigner_basis(dirs, lvals)
    (ours,) = fe.WignerDBasis([fe.Repr(lvals)])(dirs.to(cuda_device))
    err = (ours.cpu() - ref).abs().max().item()
    assert err < 3e-5, err


def _oracle_rot_to_ez(dirs, lvals):
    eps = 1e-8
    d = dirs / (torch.linalg.norm(dirs, dim=-1, keepdim=True) + eps)
    axis = torch.stack([-d[..., 1], d[..., 0], torch.zeros_like(d[..., 0])], dim=-1)
    axis = axis / (torch.linalg.norm(axis, dim=-1, keepdim=True) + eps)
    angle = torch.arccos(d[..., 2].clamp(-1 + eps, 1 - eps))
    return orc.rot(axis, angle, lvals).mT


@pytest.mark.parametrize("lvals", [[0], [1], [0, 0], [2, 2, 1], [0, 1, 2], [4, 1]])
@pytest.mark.parametrize("n", [1, 31, 33, 97, 1029])
def test_basis_ragged_groups(cuda_device, lvals, n):
    """Edge counts that leave a partial group of 32 and a dense output whose length is not a
    multiple of 4 floats, in both column orders (m-first basis, std-order rot_to_ez)."""
    g = torch.Generator().manual_seed(n)
    dirs = torch.randn(n, 3, generator=g)
    (ours,) = fe.WignerDBasis([fe.Repr(lvals)])(dirs.to(cuda_device))
    assert (ours.cpu() - orc.wigner_basis(dirs, lvals)).abs().max().item() < 3e-5
    rz = fe.WignerD(fe.Repr(lvals)).to(cuda_device).rot_to_ez(dirs.to(cuda_device))
    assert (rz.cpu() - _oracle_rot_to_ez(dirs, lvals)).abs().max().item() < 3e-5


def test_basis_high_degree_against_float64(cuda_device):
    """l up to 16 (the reference's MAX_LVALS limit) against a float64 matrix exponential."""
    g = torch.Generator().manual_seed(3)
    dirs = torch.randn(64, 3, generator=g)
    for l in (8, 12, 16):
        gens = torch.from_numpy(orc.real_generators(l, np.float64))
        (ours,) = fe.WignerDBasis([fe.Repr([l])])(dirs.to(cuda_device))
        d = dirs.double() / dirs.double().norm(dim=-1, keepdim=True)
        n = torch.hypot(d[:, 0], d[:, 1])
        th = torch.arccos(d[:, 2])
        A = (-d[:, 1] / n)[:, None, None] * gens[0] + (d[:, 0] / n)[:, None, None] * gens[1]
        D = torch.linalg.matrix_exp(th[:, None, None] * A)
        perm = torch.from_numpy(orc.m_first_perm([l]))
        err = (ours.cpu().double() - D[..., perm]).abs().max().item()
        assert err < 5e-5 * (l + 1), (l, err)


@pytest.mark.parametrize("log_bins", [False, True])
def test_binning_bit_exact(cuda_device, log_bins):
    g = torch.Generator().manual_seed(1)
    nb = 100
    lo_d, hi_d = (0.5, 8.0) if log_bins else (0.0, 10.0)
    dist = torch.cat([torch.rand(100000, generator=g) * 12 - 1,
                      torch.linspace(lo_d, hi_d, nb + 1),      # exact bin edges
                      torch.tensor([-5.0, 0.0, 100.0, lo_d, hi_d])])
    p1, p2 = orc.binning_params(nb, lo_d, hi_d, log_bins)
    lo_ref, t_ref = orc.binning(dist.numpy(), p1, p2, nb, log_bins)
    lo, t = ops.edge_binning(dist.to(cuda_device), p1, p2, nb, log_bins)
    lo, t = lo.cpu().numpy(), t.cpu().numpy()
    if log_bins:
        # logf/expf differ by an ulp between CUDA and glibc: a mismatch may only occur
        # where the normalised value sits on an integer.
        x = (np.log(np.maximum(dist.numpy().astype(np.float64), np.exp(p1))) - p1) * p2 * nb
        bad = lo != lo_ref
        assert np.all(np.abs(x[bad] - np.round(x[bad])) < 1e-4), x[bad]
        ok = ~bad
        assert np.allclose(t[ok], t_ref[ok], atol=1e-5)
    else:
        assert np.array_equal(lo, lo_ref)
        assert np.allclose(t, t_ref, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_edge_sort_bit_exact(cuda_device, dtype):
    g = torch.Generator().manual_seed(2)
    for E, K in ((0, 5), (1, 1), (1000, 7), (200000, 100), (50000, 30000)):
        keys = torch.randint(0, K, (E,), generator=g).to(dtype)
        perm, offsets, status = ops.edge_sort(keys.to(cuda_device), K)
        ref_perm = np.argsort(keys.numpy(), kind="stable")
        ref_off = np.searchsorted(np.sort(keys.numpy()), np.arange(K + 1), side="left")
        assert np.array_equal(perm.cpu().numpy(), ref_perm)
        assert np.array_equal(offsets.cpu().numpy(), ref_off)
        assert int(status.item()) == 0


def test_edge_sort_flags_out_of_range(cuda_device):
    keys = torch.tensor([0, 3, 9, 1], device=cuda_device)
    perm, offsets, status = ops.edge_sort(keys, 4)
    assert int(status.item()) == 1
    assert int(offsets[-1].item()) == 4
