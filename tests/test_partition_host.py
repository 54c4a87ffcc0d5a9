"""Host logic of the dst-range partition (no GPU): boundaries, edge ownership, the
[owned; halo] src numbering, the exchange plan and the row exchange (forward and
backward), with two and three gloo ranks on CPU."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_eq import Graph
from flash_eq.partition import dst_range_bounds, partition_graph


def _graph(n=500, k=7, seed=0):
    g = torch.Generator().manual_seed(seed)
    dst = torch.arange(n).repeat_interleave(k)
    src = torch.randint(0, n, (n * k,), generator=g)
    # uneven in-degrees: drop a random third of the edges
    keep = torch.rand(n * k, generator=g) > 0.33
    return Graph(src=src[keep], dst=dst[keep], num_nodes=n)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_partition_covers_every_edge_once_and_balances(world):
    gr = _graph()
    parts = [partition_graph(gr, world, r) for r in range(world)]
    ids = torch.cat([p.edge_ids for p in parts])
    assert torch.equal(torch.sort(ids).values, torch.arange(gr.num_edges))
    starts = [p.node_start for p in parts] + [parts[-1].node_end]
    assert starts[0] == 0 and starts[-1] == gr.num_nodes
    assert all(parts[r].node_end == parts[r + 1].node_start for r in range(world - 1))
    E = gr.num_edges
    max_deg = int(torch.bincount(gr.dst, minlength=gr.num_nodes).max())
    for p in parts:
        assert abs(p.num_edges - E / world) <= max_deg + 1
        assert torch.equal(p.dst + p.node_start, gr.dst[p.edge_ids])
        assert torch.equal(p.src_global, gr.src[p.edge_ids])
        assert int(p.dst.min()) >= 0 and int(p.dst.max()) < p.num_nodes


@pytest.mark.parametrize("world", [2, 4])
def test_halo_numbering_and_exchange_plan(world):
    gr = _graph(n=301)
    parts = [partition_graph(gr, world, r) for r in range(world)]
    x = torch.randn(gr.num_nodes, 3, 2)
    for p in parts:
        # src indexes [owned rows; halo rows], the halo in global node order
        rows = torch.cat([x[p.node_start:p.node_end], x[p.halo_global]])
        assert rows.shape[0] == p.num_src_nodes
        assert torch.equal(rows[p.src], x[p.src_global])
        assert torch.equal(torch.sort(p.halo_global).values, p.halo_global)
        assert not bool(((p.halo_global >= p.node_start) & (p.halo_global < p.node_end)).any())
        # the halo is exactly the foreign src nodes of this rank's edges
        foreign = p.src_global[(p.src_global < p.node_start) | (p.src_global >= p.node_end)]
        assert torch.equal(torch.unique(foreign), p.halo_global)
    for a in range(world):
        for b in range(world):
            assert parts[a].send_counts[b] == parts[b].recv_counts[a]
        # what a sends to b, in order, is b's halo block owned by a
        off = 0
        for b in range(world):
            c = parts[a].send_counts[b]
            sent = parts[a].send_idx[off:off + c] + parts[a].node_start
            ro = sum(parts[b].recv_counts[:a])
            assert torch.equal(sent, parts[b].halo_global[ro:ro + c])
            off += c


def test_bounds_empty_and_single():
    b = dst_range_bounds(torch.zeros(0, dtype=torch.long), 5, 3)
    assert b.tolist()[0] == 0 and b.tolist()[-1] == 5 and torch.all(b[1:] >= b[:-1])
    b = dst_range_bounds(torch.tensor([2, 2, 2]), 4, 2)
    assert b.tolist()[0] == 0 and b.tolist()[-1] == 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gr = _graph(n=257, seed=3)
        x = torch.randn(gr.num_nodes, 4, 9, generator=torch.Generator().manual_seed(5))
        p = partition_graph(gr, world, rank)
        full = p.gather_nodes(x[p.node_start:p.node_end].contiguous())
        ok = bool(torch.equal(full[p.src], x[p.src_global])) and full.shape[0] == p.num_src_nodes
        # backward: every rank's gradient of its gathered rows is summed onto the owner
        coef = torch.randn(gr.num_edges, 4, 9, generator=torch.Generator().manual_seed(6))
        xo = x[p.node_start:p.node_end].clone().requires_grad_()
        (p.gather_nodes(xo)[p.src] * coef[p.edge_ids]).sum().backward()
        want = torch.zeros_like(x).index_add_(0, gr.src, coef)[p.node_start:p.node_end]
        q.put((rank, ok, bool(torch.allclose(xo.grad, want, atol=1e-5))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_nodes_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=120) for _ in procs]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    assert all(ok and grad_ok for _, ok, grad_ok in res)


def _run_ranks(target, world, *extra, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + extra) for r in range(world)]
    for pr in procs:
        pr.start()
    res = {}
    for _ in procs:
        rank, payload = q.get(timeout=timeout)
        res[rank] = payload
    for pr in procs:
        pr.join(timeout=60)
    return res, [pr.exitcode for pr in procs]


def _subgroup_worker(rank, world, port, q):
    """Ranks 1 and 2 form a subgroup whose group ranks (0, 1) differ from their global ranks."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sub = dist.new_group([1, 2])
        if rank == 0:
            q.put((rank, True))
            return
        gr = _graph(n=211, seed=7)
        x = torch.randn(gr.num_nodes, 3, 4, generator=torch.Generator().manual_seed(8))
        me = dist.get_rank(sub)
        p = partition_graph(gr, 2, me, group=sub)
        full = p.gather_nodes(x[p.node_start:p.node_end].contiguous())
        ok = bool(torch.equal(full[p.src], x[p.src_global]))
        coef = torch.randn(gr.num_edges, 3, 4, generator=torch.Generator().manual_seed(9))
        xo = x[p.node_start:p.node_end].clone().requires_grad_()
        (p.gather_nodes(xo)[p.src] * coef[p.edge_ids]).sum().backward()
        want = torch.zeros_like(x).index_add_(0, gr.src, coef)[p.node_start:p.node_end]
        q.put((rank, ok and bool(torch.allclose(xo.grad, want, atol=1e-5))))
    finally:
        dist.destroy_process_group()


def test_gather_nodes_on_a_subgroup():
    res, codes = _run_ranks(_subgroup_worker, 3)
    assert all(c == 0 for c in codes)
    assert all(res[r] for r in range(3))


def _empty_rank_worker(rank, world, port, q):
    """Three ranks over a graph whose in-edges land on nodes 0 and 5 only: the last rank's
    range is empty (no owned node, no edge), yet it takes part in every exchange."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 6
        src = torch.tensor([1, 2, 3, 4, 5, 0, 1, 2, 3])
        dst = torch.tensor([0, 0, 0, 0, 0, 5, 5, 5, 5])
        gr = Graph(src=src, dst=dst, num_nodes=n)
        p = partition_graph(gr, world, rank)
        x = torch.randn(n, 2, 3, generator=torch.Generator().manual_seed(1))
        owned = x[p.node_start:p.node_end].contiguous()
        full = p.gather_nodes(owned)
        ok = full.shape[0] == p.num_src_nodes and bool(torch.equal(full[p.src], x[p.src_global]))
        coef = torch.randn(gr.num_edges, 2, 3, generator=torch.Generator().manual_seed(2))
        xo = owned.clone().requires_grad_()
        (p.gather_nodes(xo)[p.src] * coef[p.edge_ids]).sum().backward()
        want = torch.zeros_like(x).index_add_(0, gr.src, coef)[p.node_start:p.node_end]
        grad_ok = xo.grad is not None and bool(torch.allclose(xo.grad, want, atol=1e-6))
        q.put((rank, (p.num_nodes, ok, grad_ok)))
    finally:
        dist.destroy_process_group()


def test_gather_nodes_with_a_rank_that_owns_nothing():
    res, codes = _run_ranks(_empty_rank_worker, 3)
    assert all(c == 0 for c in codes)
    assert min(res[r][0] for r in range(3)) == 0, "the graph was meant to leave one rank empty"
    assert all(res[r][1] and res[r][2] for r in range(3))


def _leaving_rank_worker(rank, world, port, q):
    """Rank 2 leaves between two layers' exchanges (with nothing in flight); the survivors'
    next exchange must end with an error within the process-group timeout, not hang."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    gr = _graph(n=120, seed=11)
    x = torch.randn(gr.num_nodes, 2, 3, generator=torch.Generator().manual_seed(12))
    p = partition_graph(gr, world, rank)
    owned = x[p.node_start:p.node_end].contiguous()
    p.gather_nodes(owned)                          # layer 1: every rank takes part
    if rank == 2:
        q.put((rank, ("left", 0.0)))
        q.close()
        q.join_thread()
        os._exit(0)                                # leaves without a clean shutdown
    t0 = time.monotonic()
    try:
        p.gather_nodes(owned)                      # layer 2: rank 2 never answers
        q.put((rank, ("no error", time.monotonic() - t0)))
    except Exception as exc:                       # gloo: timeout or closed connection
        q.put((rank, (type(exc).__name__, time.monotonic() - t0)))
    q.close()
    q.join_thread()
    os._exit(0)


def test_survivors_see_an_error_when_a_rank_leaves():
    res, _ = _run_ranks(_leaving_rank_worker, 3, timeout=180)
    assert res[2][0] == "left"
    for r in (0, 1):
        what, waited = res[r]
        assert what != "no error", f"rank {r} finished an exchange with a missing peer"
        assert waited < 60.0, f"rank {r} waited {waited:.0f} s for the missing peer"
