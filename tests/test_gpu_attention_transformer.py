"""GPU parity of attention, pooling, the transformer block and the full model
against fixtures produced by the reference modules (tests/golden/make_golden.py).

Tolerances: softmax / pooling 1e-5 absolute (single fp32 reductions); layers
built on the edgewise linear: relative L2 1e-4.  Because LayerScale (gamma 1e-4)
makes a block's output ~ its input, the attention output is compared on its own.
"""
from __future__ import annotations

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import golden, rel_l2

pytestmark = pytest.mark.gpu


def _graph(fx, dev, n=None):
    return fe.Graph(src=fx["src"].to(dev), dst=fx["dst"].to(dev), num_nodes=n if n is not None else fx["N"])


def test_edge_attention_matches_reference(cuda_device):
    fx = golden("attention.pt")
    g = _graph(fx, cuda_device)
    Q, K, V, d = (fx[k].to(cuda_device) for k in ("Q", "K", "V", "distances"))
    for decay in (None, 3.0):
        m = fe.EquivariantEdgeAttention(num_heads=4, qk_dim=10, distance_decay_scale=decay).to(cuda_device)
        with torch.no_grad():
            m.log_scale.copy_(fx[f"log_scale_decay{decay}"])
            y = m(Q, K, V, g, d)
        assert torch.allclose(y.cpu(), fx[f"out_decay{decay}"], atol=1e-5), decay
    m1 = fe.EquivariantEdgeAttention(num_heads=1, qk_dim=40).to(cuda_device)
    with torch.no_grad():
        y1 = m1(Q.reshape(-1, 1, 40), K.reshape(-1, 1, 40), V, g)
    assert torch.allclose(y1.cpu(), fx["out_h1"], atol=1e-5)


def test_neighbor_softmax_sums_to_one(cuda_device):
    """tests/test_attention.py:77-107 of the reference."""
    attn = fe.EquivariantEdgeAttention(num_heads=2, qk_dim=36).to(cuda_device)
    g = fe.Graph.random(20, 100, device=cuda_device)
    logits = torch.randn(100, 2, device=cuda_device)
    w = attn._neighbor_softmax(logits, g.dst, 20)
    ref = orc.segment_softmax(logits.cpu(), g.dst.cpu(), 20)
    assert torch.allclose(w.cpu(), ref, atol=1e-6)
    sums = torch.zeros(20, 2, device=cuda_device).scatter_add_(0, g.dst[:, None].expand(-1, 2), w)
    has = torch.zeros(20, dtype=torch.bool, device=cuda_device)
    has[g.dst] = True
    assert torch.allclose(sums[has], torch.ones_like(sums[has]), atol=1e-5)


def test_pooling_matches_reference(cuda_device):
    fx = golden("attention.pt")
    g = _graph(fx, cuda_device)
    V = fx["V"].to(cuda_device)
    for red in ("sum", "mean", "max"):
        y = fe.GraphPooling(red)(V, g)
        assert torch.allclose(y.cpu(), fx["pool_" + red], atol=1e-5), red


def test_pooling_known_answers(cuda_device):
    """tests/test_layers.py:470-570 of the reference."""
    dev = cuda_device
    ef = torch.tensor([[[1.0, 2.0]], [[3.0, 4.0]], [[5.0, 6.0]], [[7.0, 8.0]]], device=dev)
    g = fe.Graph(src=torch.zeros(4, dtype=torch.long, device=dev), dst=torch.tensor([0, 0, 1, 1], device=dev),
                 num_nodes=2)
    assert torch.equal(fe.GraphPooling("sum")(ef, g).cpu(), torch.tensor([[[4.0, 6.0]], [[12.0, 14.0]]]))
    ef = torch.tensor([[[2.0, 4.0]], [[4.0, 8.0]], [[9.0, 3.0]]], device=dev)
    g = fe.Graph(src=torch.zeros(3, dtype=torch.long, device=dev), dst=torch.tensor([0, 0, 1], device=dev),
                 num_nodes=2)
    assert torch.equal(fe.GraphPooling("mean")(ef, g).cpu(), torch.tensor([[[3.0, 6.0]], [[9.0, 3.0]]]))
    ef = torch.tensor([[[1.0, 5.0]], [[3.0, 2.0]], [[7.0, 8.0]]], device=dev)
    assert torch.equal(fe.GraphPooling("max")(ef, g).cpu(), torch.tensor([[[3.0, 5.0]], [[7.0, 8.0]]]))
    empty = fe.Graph(src=torch.zeros(0, dtype=torch.long, device=dev), dst=torch.zeros(0, dtype=torch.long,
                     device=dev), num_nodes=3)
    for red in ("sum", "mean", "max"):
        y = fe.GraphPooling(red)(torch.zeros(0, 2, 3, device=dev), empty)
        assert y.shape == (3, 2, 3) and (y == 0).all()


def test_equivariant_attention_matches_reference(cuda_device):
    fx = golden("attention.pt")
    g = _graph(fx, cuda_device)
    rin, rout = fe.Repr([0, 1, 2], mult=8), fe.Repr([0, 1], mult=8)
    ea = fe.EquivariantAttention(rin, rout, num_heads=4, num_bins=30, distance_decay_scale=4.0)
    ea.load_state_dict(fx["ea_state"])
    ea = ea.to(cuda_device).eval()
    P, Qb = fe.WignerDBasis([rin, rout])(fx["ea_dirs"].to(cuda_device))
    x, d = fx["ea_x"].to(cuda_device), fx["distances"].to(cuda_device)
    with torch.no_grad():
        y = ea(P, Qb, x, d, g)
        y2 = ea(P, Qb, x, d, g, edge_features=fx["ea_edge_add"].to(cuda_device))
        ea.pool.reduce = "max"
        y3 = ea(P, Qb, x, d, g)
    assert rel_l2(y, fx["ea_out"]) < 1e-4
    assert rel_l2(y2, fx["ea_out_edgefeat"]) < 1e-4
    assert torch.isfinite(y3).all()


@pytest.mark.parametrize("name", ["std", "ls_none", "change"])
def test_transformer_block_matches_reference(cuda_device, name):
    fx = golden("block.pt")
    case = fx[name]
    dev = cuda_device
    coords, src, dst = fx["coords"].to(dev), fx["src"].to(dev), fx["dst"].to(dev)
    g = fe.Graph(src=src, dst=dst, num_nodes=coords.shape[0])
    rr = fe.Repr([0, 1, 2], mult=16)
    rout = fe.Repr(case["lvals_out"], mult=case["mult_out"])
    blk = fe.EquivariantTransformerBlock(rr, rout, **case["kwargs"])
    blk.load_state_dict(case["state"])
    blk = blk.to(dev).eval()
    vec = coords[src] - coords[dst]
    P, Q = fe.WignerDBasis([rr, rout])(vec)
    cap = {}
    h = blk.attn.register_forward_hook(lambda m, i, o: cap.__setitem__("attn", o))
    with torch.no_grad():
        y = blk(P, Q, case["x"].to(dev), vec.norm(dim=-1), g)
    h.remove()
    assert rel_l2(cap["attn"], case["attn_out"]) < 1e-4
    assert rel_l2(y - case["x"].to(dev) if name != "change" else y,
                  case["output"] - case["x"] if name != "change" else case["output"]) < 1e-4


def test_transformer_matches_reference(cuda_device):
    fx = golden("transformer.pt")
    dev = cuda_device
    coords, src, dst = fx["coords"].to(dev), fx["src"].to(dev), fx["dst"].to(dev)
    g = fe.Graph(src=src, dst=dst, num_nodes=coords.shape[0])
    model = fe.EquivariantTransformer(fe.Repr([0, 1], 8), fe.Repr([0, 1, 2], 16), fe.Repr([0], 4),
                                      num_layers=3, num_heads=4, max_dist=10.0)
    model.load_state_dict(fx["state"])
    model = model.to(dev).eval()
    caps = []
    hooks = [lay.register_forward_hook(lambda m, i, o: caps.append(o)) for lay in model.layers]
    with torch.no_grad():
        y = model(coords, fx["x"].to(dev), g)
    for h in hooks:
        h.remove()
    for ours, ref in zip(caps, fx["layer_outputs"]):
        assert rel_l2(ours, ref) < 1e-4
    assert rel_l2(y, fx["output"]) < 1e-4
