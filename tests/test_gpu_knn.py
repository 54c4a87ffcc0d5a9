"""GPU k-nearest-neighbour graph construction against brute force (torch.cdist + topk,
as the reference's examples build graphs): identical neighbour lists up to exact ties."""
from __future__ import annotations

import pytest
import torch

import flash_eq as fe
from flash_eq.cuda import ops

pytestmark = pytest.mark.gpu


def _brute(coords, k):
    d = torch.cdist(coords.double(), coords.double())
    d.fill_diagonal_(float("inf"))
    return d.topk(k, dim=1, largest=False)


def _walk(n, seed):
    g = torch.Generator().manual_seed(seed)
    steps = torch.randn(n, 3, generator=g)
    steps = steps / steps.norm(dim=1, keepdim=True) * 3.8
    return steps.cumsum(0)


@pytest.mark.parametrize("kind,n,k", [("cube", 4000, 16), ("cube", 3000, 32), ("walk", 6000, 16),
                                      ("walk", 500, 7), ("clustered", 2000, 12), ("tiny", 5, 8)])
def test_knn_matches_brute_force(cuda_device, kind, n, k):
    g = torch.Generator().manual_seed(3)
    if kind == "cube":
        xyz = torch.rand(n, 3, generator=g) * 40
    elif kind == "walk":
        xyz = _walk(n, 4)
    elif kind == "clustered":
        centres = torch.rand(10, 3, generator=g) * 100
        xyz = centres[torch.randint(0, 10, (n,), generator=g)] + torch.randn(n, 3, generator=g) * 0.5
    else:
        xyz = torch.rand(n, 3, generator=g)
    nbr = ops.knn(xyz.to(cuda_device), k).cpu()
    kk = min(k, n - 1)
    dist, idx = _brute(xyz, kk)
    assert (nbr[:, kk:] == -1).all()
    got = nbr[:, :kk]
    gd = (xyz.double()[got] - xyz.double()[:, None, :]).norm(dim=-1)
    # same distances in the same order (float32 vs float64 distances may order near-equal
    # pairs differently, e.g. the two chain neighbours of a random walk, both 3.8 A away) ...
    assert torch.allclose(gd, dist, rtol=1e-6, atol=1e-6)
    # ... and the same neighbour sets, except where the k-th distance ties the next one
    if n - 1 > kk:
        dnext = _brute(xyz, kk + 1)[0][:, -1]
        tie = (dnext - dist[:, -1]).abs() <= 1e-5 * dist[:, -1].clamp(min=1e-6)
    else:
        tie = torch.zeros(n, dtype=torch.bool)
    sets_equal = (got.sort(dim=1).values == idx.sort(dim=1).values).all(dim=1)
    assert bool((sets_equal | tie).all())


def test_knn_graph_matches_cdist_convention(cuda_device):
    xyz = torch.rand(2000, 3, generator=torch.Generator().manual_seed(5)) * 30
    gr = fe.Graph.knn(xyz.to(cuda_device), 16)
    _, idx = _brute(xyz, 16)
    assert gr.num_edges == 2000 * 16
    assert torch.equal(gr.dst.cpu(), torch.arange(2000).repeat_interleave(16))
    assert (gr.src.cpu().view(2000, 16).sort(dim=1).values == idx.sort(dim=1).values).float().mean() > 0.999


def test_knn_cell_size_does_not_change_result(cuda_device):
    xyz = (torch.rand(3000, 3, generator=torch.Generator().manual_seed(6)) * 50).to(cuda_device)
    a = ops.knn(xyz, 16)
    for cell in (0.9, 3.0, 25.0):
        assert torch.equal(ops.knn(xyz, 16, cell=cell), a)
