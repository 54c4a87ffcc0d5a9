"""Fused attention pooling at the transformer workloads' row shapes (64 channels x 9, 8 heads;
32 x 16; 64 x 4) against the CPU restatement of the reference (attention.py:92-167,
pooling.py:21-57): Q / K from node rows, online softmax over each destination's in-edges, the
weighted V rows summed (or averaged).  Covers the warp-per-destination kernel these shapes
take: split K rows (partitioned graphs), the distance decay, mean pooling, destinations
without in-edges and a bad src index.  Tolerance 1e-5 relative L2 (float32 throughout)."""
from __future__ import annotations

import pytest
import torch

import feq_oracle as orc
from conftest import rel_l2
from flash_eq.cuda import ops

pytestmark = pytest.mark.gpu


def _graph(N, E, gen, empty=7):
    src = torch.randint(0, N, (E,), generator=gen)
    dst = torch.randint(0, N - empty, (E,), generator=gen)        # the last nodes get no in-edge
    return src, dst


@pytest.mark.parametrize("C,d,H", [(64, 9, 8), (32, 16, 4), (64, 4, 2), (32, 9, 1)])
@pytest.mark.parametrize("decay,reduce,split", [(None, "sum", False), (3.0, "mean", False), (2.0, "sum", True)])
def test_attn_pool_matches_oracle(cuda_device, C, d, H, decay, reduce, split):
    gen = torch.Generator().manual_seed(C * d + H)
    N, E = 900, 20000
    src, dst = _graph(N, E, gen)
    qk = torch.randn(N, 2 * C, d, generator=gen)
    V = torch.randn(E, C, d, generator=gen)
    dist = torch.rand(E, generator=gen) * 6
    scale = 0.3
    perm, offsets, status = ops.edge_sort(dst.to(cuda_device), N)
    kwargs = {}
    q_in = qk.to(cuda_device)
    if split:
        q_in = qk[:, :C].contiguous().to(cuda_device)
        kwargs["k"] = qk[:, C:].contiguous().to(cuda_device)
    out = ops.attn_pool(q_in, V.to(cuda_device), src.to(cuda_device), dist.to(cuda_device), perm, offsets, N, H,
                        scale, decay, reduce, **kwargs)
    torch.cuda.synchronize()
    Qe = qk[:, :C][dst].reshape(E, H, -1)
    Ke = qk[:, C:][src].reshape(E, H, -1)
    w = orc.edge_attention(Qe, Ke, V, dst, N, torch.tensor(scale), H, dist if decay else None, decay)
    ref = orc.pool(w, dst, N, reduce)
    assert rel_l2(out, ref) < 1e-5
    assert out[N - 7:].abs().max().item() == 0.0


def test_attn_pool_bad_src_sets_status(cuda_device):
    gen = torch.Generator().manual_seed(5)
    N, E, C, d, H = 300, 4000, 64, 9, 8
    src, dst = _graph(N, E, gen)
    src[11] = N + 3
    qk = torch.randn(N, 2 * C, d, generator=gen)
    V = torch.randn(E, C, d, generator=gen)
    perm, offsets, _ = ops.edge_sort(dst.to(cuda_device), N)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = ops.attn_pool(qk.to(cuda_device), V.to(cuda_device), src.to(cuda_device), None, perm, offsets, N, H, 0.3,
                        None, "sum", status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("decay", [None, 2.0])
def test_attn_pool_hub_destination(cuda_device, decay):
    """One destination with 300 in-edges (its edge ids arrive in batches of 32), the others
    with one edge or none: the batched index loads and the row ring across batch boundaries."""
    gen = torch.Generator().manual_seed(17)
    N, C, d, H = 40, 64, 9, 8
    hub = torch.full((300,), 3, dtype=torch.int64)
    single = torch.arange(10, 30)
    dst = torch.cat([hub, single])
    E = dst.numel()
    src = torch.randint(0, N, (E,), generator=gen)
    qk = torch.randn(N, 2 * C, d, generator=gen)
    V = torch.randn(E, C, d, generator=gen)
    dist = torch.rand(E, generator=gen) * 6
    perm, offsets, _ = ops.edge_sort(dst.to(cuda_device), N)
    out = ops.attn_pool(qk.to(cuda_device), V.to(cuda_device), src.to(cuda_device), dist.to(cuda_device), perm,
                        offsets, N, H, 0.25, decay, "sum")
    torch.cuda.synchronize()
    Qe = qk[:, :C][dst].reshape(E, H, -1)
    Ke = qk[:, C:][src].reshape(E, H, -1)
    w = orc.edge_attention(Qe, Ke, V, dst, N, torch.tensor(0.25), H, dist if decay else None, decay)
    ref = orc.pool(w, dst, N, "sum")
    assert rel_l2(out, ref) < 1e-5
