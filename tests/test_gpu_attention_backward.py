"""GPU parity of the attention / pooling backward and of training the attention layer,
the transformer block and the transformer.

The checker is the reference's own formulation differentiated by PyTorch autograd in
float64 on the CPU: ``orc.edge_attention`` / ``orc.segment_softmax`` / ``orc.pool``
restate flash_eq/layers/attention.py:72-167 and pooling.py:21-57 (pinned to the
reference's outputs by the golden fixtures), and the edgewise linear's block-diagonal
step uses the float64 C restatement of the reference's forward and backward kernels.
Each result is also computed by the same reference formulation in float32 on the CPU.
Tolerance per output / gradient (relative L2 against float64): 5e-5 for the operators
and 1e-4 for layers that include the edgewise linear (bf16x3 tensor-core mix), or three
times the float32 reference's own error where that is larger -- some gradients are
ill-conditioned sums (a scalar log_scale gradient, gradients through a layer norm of
nearly constant inputs), and there even the float32 reference misses float64 by 1e-3.
"""
from __future__ import annotations

import copy

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import attention_autograd as aag
from flash_eq.layers.pooling import pool_edges
from flash_eq.partition import PartitionedGraph

pytestmark = pytest.mark.gpu

OP_TOL = 5e-5
LAYER_TOL = 1e-4


def _close(got, ref64, ref32, tol, what=""):
    err, base = rel_l2(got, ref64), rel_l2(ref32, ref64)
    assert err < max(tol, 3.0 * base), f"{what}: {err:.2e} (float32 reference {base:.2e})"


def _graph_edges(N, E, seed, hub=True, isolated=5):
    """Random edges; node 0 is a hub with 100 extra in-edges (several 32-edge chunks); the
    last ``isolated`` nodes have no in-edges; nodes 0 and 1 have no out-edges."""
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(2, N, (E,), generator=g)
    dst = torch.randint(0, N - isolated, (E,), generator=g)
    if hub:
        src = torch.cat([src, torch.randint(2, N, (100,), generator=g)])
        dst = torch.cat([dst, torch.zeros(100, dtype=torch.long)])
    return src, dst


def _ref_attn_pool(qk, v, src, dst, N, H, log_scale, dist, decay, reduce, k=None):
    C = qk.shape[1] // 2 if k is None else qk.shape[1]
    E = src.shape[0]
    Qe = (qk[:, :C] if k is None else qk)[dst].reshape(E, H, -1)
    Ke = (qk[:, C:] if k is None else k)[src].reshape(E, H, -1)
    weighted = orc.edge_attention(Qe, Ke, v, dst, N, log_scale.exp(), H, dist, decay)
    return orc.pool(weighted, dst, N, reduce)


@pytest.mark.parametrize("split_k", [False, True])
@pytest.mark.parametrize("decay", [None, 2.5])
@pytest.mark.parametrize("reduce", ["sum", "mean"])
@pytest.mark.parametrize("H", [1, 2, 4])
def test_attn_pool_backward_matches_autograd_of_reference(cuda_device, H, reduce, decay, split_k):
    dev = cuda_device
    N, E, C, d, Cv, dv = 60, 900, 8, 9, 12, 4
    src, dst = _graph_edges(N, E, seed=H + 7 * (decay is not None))
    E = src.shape[0]
    g = torch.Generator().manual_seed(11)
    Nsrc = N + 13 if split_k else N
    qk = torch.randn(N, C if split_k else 2 * C, d, generator=g)
    kk = torch.randn(Nsrc, C, d, generator=g) if split_k else None
    v = torch.randn(E, Cv, dv, generator=g)
    dist = torch.rand(E, generator=g) * 8 + 0.5
    log_scale = torch.tensor((C // H * d) ** -0.5).log() + 0.3
    go = torch.randn(N, Cv, dv, generator=g)

    if split_k:
        graph = PartitionedGraph(src=src.to(dev), dst=dst.to(dev), num_nodes=N, num_src_nodes=Nsrc)
    else:
        graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)
    leaves = [t.to(dev).requires_grad_() for t in (qk, v, dist, log_scale)]
    kg = kk.to(dev).requires_grad_() if split_k else None
    scale = float(leaves[3].detach().exp())
    out = aag.attn_pool(leaves[0], leaves[1], leaves[2], leaves[3], graph, H, scale, decay, reduce, k=kg)
    out.backward(go.to(dev))

    refs = {}
    for dt in (torch.float64, torch.float32):
        rl = [t.to(dt).requires_grad_() for t in (qk, v, dist, log_scale)]
        rk = kk.to(dt).requires_grad_() if split_k else None
        ref = _ref_attn_pool(rl[0], rl[1], src, dst, N, H, rl[3], rl[2], decay, reduce, k=rk)
        ref.backward(go.to(dt))
        refs[dt] = (ref.detach(), rl, rk)
    (r64, l64, k64), (r32, l32, k32) = refs[torch.float64], refs[torch.float32]
    _close(out.detach(), r64, r32, OP_TOL, "out")
    for i, name in enumerate(("qk", "v", "dist", "log_scale")):
        if name == "dist" and decay is None:
            assert leaves[i].grad is None
            continue
        _close(leaves[i].grad, l64[i].grad, l32[i].grad, OP_TOL, name)
    if split_k:
        _close(kg.grad, k64.grad, k32.grad, OP_TOL, "k")


@pytest.mark.parametrize("Cv,dv,H", [(64, 25, 8), (64, 9, 8), (32, 16, 4), (7, 9, 1)])
def test_attn_pool_forward_row_sizes(cuda_device, Cv, dv, H):
    """Forward pooling across V row sizes: chunks of 9 to 32 edges through shared memory
    (bulk-copied rows), and rows that do not split into whole float4 head slices (7 x 9)."""
    dev = cuda_device
    N, E, C, d = 50, 600, 16, 9
    src, dst = _graph_edges(N, E, seed=Cv + dv)
    E = src.shape[0]
    g = torch.Generator().manual_seed(5)
    qk = torch.randn(N, 2 * C, d, generator=g)
    v = torch.randn(E, Cv, dv, generator=g)
    log_scale = torch.tensor(-1.2)
    graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)
    out = aag.attn_pool(qk.to(dev), v.to(dev), None, log_scale.to(dev), graph, H, float(log_scale.exp()), None,
                        "sum")
    r64 = _ref_attn_pool(qk.double(), v.double(), src, dst, N, H, log_scale.double(), None, None, "sum")
    r32 = _ref_attn_pool(qk, v, src, dst, N, H, log_scale, None, None, "sum")
    _close(out, r64, r32, OP_TOL, "out")


def test_attn_pool_backward_deterministic_and_empty(cuda_device):
    dev = cuda_device
    N, E = 40, 700
    src, dst = _graph_edges(N, E, seed=3)
    graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)
    g = torch.Generator().manual_seed(1)
    qk = torch.randn(N, 16, 9, generator=g).to(dev)
    v = torch.randn(src.shape[0], 8, 9, generator=g).to(dev)
    go = torch.randn(N, 8, 9, generator=g).to(dev)
    ls = torch.tensor(-1.0, device=dev)
    grads = []
    for _ in range(2):
        a, b, c = (t.clone().requires_grad_() for t in (qk, v, ls))
        aag.attn_pool(a, b, None, c, graph, 2, float(c.detach().exp()), None, "sum").backward(go)
        grads.append((a.grad, b.grad, c.grad))
    for x, y in zip(*grads):
        assert torch.equal(x, y)
    # a graph without edges: zero output, zero gradients
    empty = fe.Graph(src=torch.zeros(0, dtype=torch.long, device=dev), dst=torch.zeros(0, dtype=torch.long,
                     device=dev), num_nodes=N)
    a = qk.clone().requires_grad_()
    b = torch.zeros(0, 8, 9, device=dev, requires_grad=True)
    y = aag.attn_pool(a, b, None, ls, empty, 2, 0.5, None, "mean")
    y.backward(go)
    assert (y == 0).all() and (a.grad == 0).all()


@pytest.mark.parametrize("decay", [None, 3.0])
@pytest.mark.parametrize("H", [1, 4])
def test_edge_attention_backward(cuda_device, H, decay):
    dev = cuda_device
    N, E, D = 50, 800, 20
    src, dst = _graph_edges(N, E, seed=5)
    E = src.shape[0]
    g = torch.Generator().manual_seed(2)
    Q, K = torch.randn(E, H, D, generator=g), torch.randn(E, H, D, generator=g)
    V = torch.randn(E, 8, 5, generator=g)
    dist = torch.rand(E, generator=g) * 6 + 0.3
    go = torch.randn(E, 8, 5, generator=g)
    graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)
    m = fe.EquivariantEdgeAttention(num_heads=H, qk_dim=D, distance_decay_scale=decay).to(dev)
    xs = [t.to(dev).requires_grad_() for t in (Q, K, V, dist)]
    y = m(xs[0], xs[1], xs[2], graph, xs[3])
    y.backward(go.to(dev))
    refs = {}
    for dt in (torch.float64, torch.float32):
        rs = [t.to(dt).requires_grad_() for t in (Q, K, V, dist)]
        ls = m.log_scale.detach().cpu().to(dt).requires_grad_()
        orc.edge_attention(rs[0], rs[1], rs[2], dst, N, ls.exp(), H, rs[3], decay).backward(go.to(dt))
        refs[dt] = rs + [ls]
    for i, name in enumerate("QKVd"):
        if name == "d" and decay is None:
            assert xs[i].grad is None
            continue
        _close(xs[i].grad, refs[torch.float64][i].grad, refs[torch.float32][i].grad, OP_TOL, name)
    _close(m.log_scale.grad, refs[torch.float64][4].grad, refs[torch.float32][4].grad, OP_TOL, "log_scale")


def test_neighbor_softmax_backward(cuda_device):
    dev = cuda_device
    N, E = 30, 400
    src, dst = _graph_edges(N, E, seed=9)
    lg = torch.randn(src.shape[0], 3, generator=torch.Generator().manual_seed(4))
    gw = torch.randn(src.shape[0], 3, generator=torch.Generator().manual_seed(5))
    attn = fe.EquivariantEdgeAttention(num_heads=3, qk_dim=3).to(dev)
    x = lg.to(dev).requires_grad_()
    attn._neighbor_softmax(x, dst.to(dev), N).backward(gw.to(dev))
    r = lg.double().requires_grad_()
    orc.segment_softmax(r, dst, N).backward(gw.double())
    r32 = lg.clone().requires_grad_()
    orc.segment_softmax(r32, dst, N).backward(gw)
    _close(x.grad, r.grad, r32.grad, OP_TOL, "logits")


@pytest.mark.parametrize("weighted", [False, True])
@pytest.mark.parametrize("reduce", ["sum", "mean", "max"])
def test_pooling_backward(cuda_device, reduce, weighted):
    dev = cuda_device
    N, E, H = 40, 600, 2
    src, dst = _graph_edges(N, E, seed=13)
    E = src.shape[0]
    g = torch.Generator().manual_seed(8)
    x = torch.randn(E, 6, 5, generator=g)
    # ties for max: the first two in-edges of every node get the same row
    order = torch.argsort(dst, stable=True)
    first = torch.ones(E, dtype=torch.bool)
    first[1:] = dst[order[1:]] != dst[order[:-1]]
    pos = torch.nonzero(first).flatten()
    pos = pos[pos + 1 < E]
    pos = pos[dst[order[pos]] == dst[order[pos + 1]]]
    x[order[pos + 1]] = x[order[pos]]
    w = torch.rand(E, H, generator=g) + 0.5 if weighted else None
    go = torch.randn(N, 6, 5, generator=g)
    graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)
    xg = x.to(dev).requires_grad_()
    wg = w.to(dev).requires_grad_() if weighted else None
    y = pool_edges(xg, graph, reduce, weights=wg)
    y.backward(go.to(dev))
    refs = {}
    for dt in (torch.float64, torch.float32):
        xr = x.to(dt).requires_grad_()
        wr = w.to(dt).requires_grad_() if weighted else None
        rows = (xr.view(E, H, 3, 5) * wr.view(E, H, 1, 1)).view(E, 6, 5) if weighted else xr
        ref = orc.pool(rows, dst, N, reduce)
        ref.backward(go.to(dt))
        refs[dt] = (ref.detach(), xr, wr)
    (r64, x64, w64), (r32, x32, w32) = refs[torch.float64], refs[torch.float32]
    _close(y.detach(), r64, r32, OP_TOL, "out")
    _close(xg.grad, x64.grad, x32.grad, OP_TOL, "rows")
    if weighted:
        _close(wg.grad, w64.grad, w32.grad, OP_TOL, "weights")


# ---------------------------------------------------------------------------
# Layers: the float64 CPU reference composition
# ---------------------------------------------------------------------------
class _OracleBlockDiagonal(torch.autograd.Function):
    """block_diagonal_cuda on the CPU: the C restatement of the reference's forward
    (block_diagonal.cu:558-733; float32 or float64 like the inputs) and backward
    (block_diagonal.cu:747-1161; float64, returned in the inputs' dtype)."""

    @staticmethod
    def forward(ctx, f, table, dist, cfg):
        ctx.save_for_backward(f, table, dist)
        ctx.cfg = cfg
        return orc.block_diagonal_fwd(f, table, dist, *cfg)

    @staticmethod
    def backward(ctx, go):
        f, table, dist = ctx.saved_tensors
        gf, gt, gd = orc.block_diagonal_bwd(go, f, table, dist, *ctx.cfg)
        return gf.to(f.dtype), gt.to(table.dtype), gd.to(dist.dtype), None


def _ref_attention(att, P, Q, x, dist, src, dst, N, edge_features=None):
    """EquivariantAttention.forward as the reference writes it (attention.py:271-314) on
    the CPU; ``att`` is a CPU copy of the layer in the reference's dtype."""
    mult = att.in_repr.mult
    E = src.shape[0]
    qk = att.linear_qk(att.norm_qk(x))
    Qe = qk[:, :mult][dst].reshape(E, att.num_heads, -1)
    Ke = qk[:, mult:][src].reshape(E, att.num_heads, -1)
    f = x[src]
    if edge_features is not None:
        f = f + edge_features
    lv = att.linear_v
    rw = lv.radial_weights
    p1, p2 = rw.binning_params()
    cfg = (list(lv._lin), list(lv._lout), lv.solid_harmonic_scale, p1, p2, rw.num_bins, rw.log)
    V = torch.bmm(_OracleBlockDiagonal.apply(torch.bmm(f, P), rw(), dist, cfg), Q.mT)
    w = orc.edge_attention(Qe, Ke, V, dst, N, att.attention.log_scale.exp(), att.num_heads, dist,
                           att.attention.distance_decay_scale)
    return orc.pool(w, dst, N, att.pool.reduce)


def _cpu_ref(module, dtype):
    ref = copy.deepcopy(module).cpu().to(dtype)
    for mod in ref.modules():
        if isinstance(mod, fe.EquivariantAttention):
            mod.forward = (lambda m: lambda P, Q, x, d, graph, edge_features=None: _ref_attention(
                m, P, Q, x, d, graph.src.cpu(), graph.dst.cpu(), graph.num_nodes, edge_features))(mod)
    return ref


def _compare_grads(gpu_mod, refs, tol):
    bad = []
    for (n, a), (_, b), (_, c) in zip(gpu_mod.named_parameters(), refs[torch.float64].named_parameters(),
                                      refs[torch.float32].named_parameters()):
        if b.grad is None:
            assert a.grad is None or not a.grad.any(), n
            continue
        assert a.grad is not None, n
        err, base = rel_l2(a.grad, b.grad), rel_l2(c.grad, b.grad)
        if err >= max(tol, 3.0 * base):
            bad.append((n, err, base))
    assert not bad, bad


def _setup(seed, N=48, k=10, lin=(0, 1, 2), mult=8):
    g = torch.Generator().manual_seed(seed)
    coords = torch.randn(N, 3, generator=g) * 2.0
    dst = torch.arange(N).repeat_interleave(k)
    src = torch.randint(0, N, (N * k,), generator=g)
    keep = src != dst
    src, dst = src[keep], dst[keep]
    rin = fe.Repr(list(lin), mult=mult)
    x = torch.randn(N, mult, rin.dim(), generator=g)
    return g, coords, src, dst, rin, x


@pytest.mark.parametrize("heads,decay,edge_feats", [(1, None, False), (2, 2.0, True), (4, None, False)])
def test_attention_layer_training_gradients(cuda_device, heads, decay, edge_feats):
    dev = cuda_device
    torch.manual_seed(0)
    g, coords, src, dst, rin, x = _setup(1)
    N, E = x.shape[0], src.shape[0]
    rout = fe.Repr([0, 1], mult=12)
    layer = fe.EquivariantAttention(rin, rout, num_heads=heads, distance_decay_scale=decay).to(dev)
    with torch.no_grad():
        layer.attention.log_scale.add_(0.7)      # make the softmax non-trivial
    vec = coords[src] - coords[dst]
    dist = vec.norm(dim=-1)
    P, Q = fe.WignerDBasis([rin, rout])(vec.to(dev))
    ef = torch.randn(E, rin.mult, rin.dim(), generator=g) if edge_feats else None
    go = torch.randn(N, rout.mult, rout.dim(), generator=g)
    graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)

    xg = x.to(dev).requires_grad_()
    dg = dist.to(dev).requires_grad_()
    eg = ef.to(dev).requires_grad_() if edge_feats else None
    y = layer(P, Q, xg, dg, graph, edge_features=eg)
    y.backward(go.to(dev))

    refs, res = {}, {}
    for dt in (torch.float64, torch.float32):
        ref = refs[dt] = _cpu_ref(layer, dt)
        xr = x.to(dt).requires_grad_()
        dr = dist.to(dt).requires_grad_()
        er = ef.to(dt).requires_grad_() if edge_feats else None
        yr = ref(P.to(dt).cpu(), Q.to(dt).cpu(), xr, dr, graph, edge_features=er)
        yr.backward(go.to(dt))
        res[dt] = (yr.detach(), xr, dr, er)
    (y64, x64, d64, e64), (y32, x32, d32, e32) = res[torch.float64], res[torch.float32]
    _close(y.detach(), y64, y32, LAYER_TOL, "out")
    _close(xg.grad, x64.grad, x32.grad, LAYER_TOL, "x")
    _close(dg.grad, d64.grad, d32.grad, LAYER_TOL, "distances")
    if edge_feats:
        _close(eg.grad, e64.grad, e32.grad, LAYER_TOL, "edge_features")
    _compare_grads(layer, refs, LAYER_TOL)


def test_transformer_block_training_gradients(cuda_device):
    dev = cuda_device
    torch.manual_seed(1)
    g, coords, src, dst, rin, x = _setup(2, lin=(0, 1, 2), mult=8)
    N = x.shape[0]
    block = fe.EquivariantTransformerBlock(rin, rin, num_heads=2, layer_scale_init=0.3).to(dev)
    vec = coords[src] - coords[dst]
    dist = vec.norm(dim=-1)
    P = fe.WignerDBasis([rin])(vec.to(dev))[0]
    go = torch.randn(N, rin.mult, rin.dim(), generator=g)
    graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)
    xg = x.to(dev).requires_grad_()
    block(P, P, xg, dist.to(dev), graph).backward(go.to(dev))
    refs, xs = {}, {}
    for dt in (torch.float64, torch.float32):
        ref = refs[dt] = _cpu_ref(block, dt)
        xr = xs[dt] = x.to(dt).requires_grad_()
        Pc = P.to(dt).cpu()
        ref(Pc, Pc, xr, dist.to(dt), graph).backward(go.to(dt))
    _close(xg.grad, xs[torch.float64].grad, xs[torch.float32].grad, LAYER_TOL, "x")
    _compare_grads(block, refs, LAYER_TOL)


def _ref_transformer_loss(ref, bases, dist, x, graph, target):
    """EquivariantTransformer.forward (transformer.py:389-431) with precomputed bases."""
    m_in, m_hid, m_out = bases
    h = x
    for i, layer in enumerate(ref.layers):
        P = m_in if i == 0 else m_hid
        Q = m_out if i == len(ref.layers) - 1 else m_hid
        h = layer(P, Q, h, dist, graph)
    return ((ref.final_norm(h) - target) ** 2).mean()


def test_transformer_training_gradients_and_step(cuda_device):
    """Two-layer EquivariantTransformer: parameter gradients against the reference
    composition, then Adam steps lower the loss."""
    dev = cuda_device
    torch.manual_seed(2)
    g, coords, src, dst, rin, x = _setup(3, lin=(0, 1), mult=6)
    N = x.shape[0]
    hid, rout = fe.Repr([0, 1, 2], mult=8), fe.Repr([0, 1], mult=4)
    model = fe.EquivariantTransformer(rin, hid, rout, num_layers=2, num_heads=2, layer_scale_init=0.3).to(dev)
    graph = fe.Graph(src=src.to(dev), dst=dst.to(dev), num_nodes=N)
    target = torch.randn(N, rout.mult, rout.dim(), generator=g)
    loss = ((model(coords.to(dev), x.to(dev), graph) - target.to(dev)) ** 2).mean()
    loss.backward()

    vec = coords[src] - coords[dst]
    bases = fe.WignerDBasis([rin, hid, rout])(vec.to(dev))
    refs, losses = {}, {}
    for dt in (torch.float64, torch.float32):
        ref = refs[dt] = _cpu_ref(model, dt)
        lr = _ref_transformer_loss(ref, [M.to(dt).cpu() for M in bases], vec.norm(dim=-1).to(dt), x.to(dt), graph,
                                   target.to(dt))
        lr.backward()
        losses[dt] = lr.item()
    assert abs(loss.item() - losses[torch.float64]) <= LAYER_TOL * abs(losses[torch.float64])
    _compare_grads(model, refs, LAYER_TOL)

    opt = torch.optim.Adam(model.parameters(), lr=3e-3)
    first = None
    for _ in range(15):
        opt.zero_grad()
        l = ((model(coords.to(dev), x.to(dev), graph) - target.to(dev)) ** 2).mean()
        l.backward()
        opt.step()
        first = l.item() if first is None else first
    assert l.item() < first
