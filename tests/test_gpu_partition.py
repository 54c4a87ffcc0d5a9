"""dst-range partitioned EquivariantTransformer on 2 GPUs (per layer an NCCL halo exchange,
all_to_all_single of just the src-side rows each rank reads) against the same model run whole
on one GPU.  Child processes, one per
GPU; NVLS off.  Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _walk_graph(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    steps = torch.randn(n, 3, generator=g)
    coords = torch.cumsum(3.8 * steps / steps.norm(dim=1, keepdim=True), 0)
    d = torch.cdist(coords, coords)
    d.fill_diagonal_(float("inf"))
    nbr = d.topk(k, dim=1, largest=False).indices
    return coords, nbr.reshape(-1), torch.arange(n).repeat_interleave(k)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    import flash_eq as fe
    from flash_eq.partition import partition_graph

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        coords, src, dst = _walk_graph(3000, 16, seed=4)
        x = torch.randn(3000, 16, 9, generator=torch.Generator().manual_seed(1))
        torch.manual_seed(7)
        model = fe.EquivariantTransformer(fe.Repr([0, 1, 2], 16), fe.Repr([0, 1, 2], 16), fe.Repr([0, 1, 2], 16),
                                          num_layers=2, num_heads=4).to(dev).eval()
        graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=3000)
        with torch.no_grad():
            whole = model(coords.to(dev), x.to(dev), graph)
            part = partition_graph(graph, world, rank)
            y = model(coords.to(dev), x[part.node_start:part.node_end].to(dev), part)
        torch.cuda.synchronize()
        ref = whole[part.node_start:part.node_end]
        err = float((y - ref).norm() / ref.norm().clamp_min(1e-30))
        q.put((rank, err, part.num_edges, graph.num_edges))
    except Exception as exc:                       # report, then leave the group cleanly
        q.put((rank, repr(exc), 0, 0))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_partitioned_transformer_matches_whole_graph():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert sum(r[2] for r in res) == res[0][3]
    for rank, err, _, _ in res:
        assert isinstance(err, float), err
        assert err < 1e-5, (rank, err)
