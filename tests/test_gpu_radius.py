"""Graph.radius (GPU cell lists) against brute force: the edge set must be identical, in
(src, dst) order, with the cut-off decided by the same float32 arithmetic
((dx*dx + dy*dy) + dz*dz < r*r, every operation rounded separately)."""
from __future__ import annotations

import pytest
import torch

import bench
import flash_eq as fe

pytestmark = pytest.mark.gpu


def brute(coords, r, batch=None, loop=False, chunk=2048):
    """Every ordered pair (i, j) closer than r, computed on the CPU, (src, dst) order."""
    c = coords.float().cpu()
    n = c.shape[0]
    r2 = torch.tensor(r, dtype=torch.float32) * torch.tensor(r, dtype=torch.float32)
    srcs, dsts = [], []
    for s in range(0, n, chunk):
        a = c[s:s + chunk]
        dx = c[None, :, 0] - a[:, None, 0]
        dy = c[None, :, 1] - a[:, None, 1]
        dz = c[None, :, 2] - a[:, None, 2]
        d2 = (dx * dx + dy * dy) + dz * dz
        m = d2 < r2
        if batch is not None:
            b = batch.cpu()
            m &= b[s:s + chunk, None] == b[None, :]
        if not loop:
            idx = torch.arange(s, min(n, s + chunk))
            m[torch.arange(idx.numel()), idx] = False
        i, j = torch.nonzero(m, as_tuple=True)
        srcs.append(i + s)
        dsts.append(j)
    return torch.cat(srcs), torch.cat(dsts)


def _check(coords, r, batch=None, loop=False):
    g = fe.Graph.radius(coords.cuda(), r, batch=None if batch is None else batch.cuda(), loop=loop)
    s_ref, d_ref = brute(coords, r, batch, loop)
    assert torch.equal(g.src.cpu(), s_ref) and torch.equal(g.dst.cpu(), d_ref)
    return g


def test_radius_config3_batch_matches_bench_construction(cuda_device):
    """The batched molecule graphs of the config-3 workload: 256 graphs x 30 nodes, r = 5."""
    wl = bench.make_block_workload(bench.BLOCK_SEED, "cpu")
    coords = wl["coords"]
    batch = torch.arange(bench.BLOCK_GRAPHS).repeat_interleave(bench.BLOCK_NODES)
    g = _check(coords, bench.BLOCK_RADIUS, batch)
    # the same edges, in the same order, as the workload's dense CPU construction
    assert torch.equal(g.src.cpu(), wl["src"]) and torch.equal(g.dst.cpu(), wl["dst"])


@pytest.mark.parametrize("n,r", [(8000, 2.5), (3000, 7.0), (1, 1.0), (2, 100.0)])
def test_radius_single_graph(cuda_device, n, r):
    gen = torch.Generator().manual_seed(n)
    coords = torch.rand(n, 3, generator=gen) * 40.0 - 20.0
    _check(coords, r)


def test_radius_duplicates_loops_and_exact_cutoff(cuda_device):
    coords = torch.tensor([[0.0, 0.0, 0.0], [0.0, 0.0, 0.0], [1.0, 0.0, 0.0], [0.0, 2.0, 0.0],
                           [5.0, 5.0, 5.0], [5.0, 5.0, 6.0]])
    g = _check(coords, 1.0)                      # |(1,0,0)| == r exactly: not an edge
    assert g.num_edges == 2                      # the duplicate pair, both directions
    _check(coords, 1.0, loop=True)
    _check(coords, 1.0000001)


def test_radius_batches_do_not_mix_and_may_be_empty(cuda_device):
    gen = torch.Generator().manual_seed(3)
    coords = torch.randn(500, 3, generator=gen)
    batch = torch.randint(0, 40, (500,), generator=gen) * 3          # gaps: empty graph ids
    batch, order = torch.sort(batch)
    _check(coords[order], 1.5, batch)
    _check(coords, 1.5, torch.randint(0, 7, (500,), generator=gen))  # unsorted batch ids
