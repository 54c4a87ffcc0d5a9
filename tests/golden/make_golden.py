"""Generate the golden fixtures under tests/golden/ by running the REFERENCE.

Run where the reference tree is available ($FEQ_REFERENCE_ROOT, else a directory
named ``reference`` beside this repository):

    python tests/golden/make_golden.py [--ref PATH]

What it does:
* stubs ``sphericart`` / ``sphericart.torch`` (imported at module level by the
  reference's out-of-scope S^2 code, flash_eq/spherical/harmonics.py:13; not on
  the edge-message path) so ``import flash_eq`` works on a CPU-only box;
* replaces ``flash_eq.layers.linear.block_diagonal_cuda`` (the one op with no
  CPU implementation in the reference, flash_eq/cuda/block_diagonal.py:46-55)
  with the CPU restatement in ``oracle/`` -- everything else is the reference's
  own code running unmodified;
* saves seeded inputs, reference ``state_dict``s and reference outputs as small
  ``.pt`` fixtures.  The GPU parity tests load those state dicts into the B200
  modules and compare.

The fixtures are committed; this script is only needed to regenerate them.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))


def import_reference(ref_root: str):
    for name in ("sphericart", "sphericart.torch"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.path.insert(0, ref_root)
    import flash_eq  # noqa: F401  (the reference)

    assert os.path.abspath(flash_eq.__file__).startswith(os.path.abspath(ref_root)), flash_eq.__file__
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import feq_oracle

    def cpu_block_diagonal(features, radial_table, distances, product_repr, bin_param1, bin_param2,
                           num_bins, log_bins=False, sh_scale=0.1):
        # Same contract as flash_eq.cuda.block_diagonal.block_diagonal_cuda (:206-274).
        lin = product_repr.rep1.lvals.tolist()
        lout = product_repr.rep2.lvals.tolist()
        if features.shape[0] == 0:
            return torch.zeros(0, radial_table.size(1), product_repr.rep2.dim(), dtype=features.dtype)
        return feq_oracle.block_diagonal_fwd(features.contiguous(), radial_table.contiguous(),
                                             distances.to(features.dtype), lin, lout, sh_scale,
                                             bin_param1, bin_param2, num_bins, log_bins)

    import flash_eq.layers.linear as ref_linear

    ref_linear.block_diagonal_cuda = cpu_block_diagonal
    return flash_eq, feq_oracle


def knn_graph(coords: torch.Tensor, k: int, batch: torch.Tensor | None = None):
    """src -> dst k-nearest-neighbour graph (no self loops); src ranges over dst's neighbours."""
    n = coords.shape[0]
    d = torch.cdist(coords.double(), coords.double())
    d.fill_diagonal_(float("inf"))
    if batch is not None:
        d[batch[:, None] != batch[None, :]] = float("inf")
    nbr = d.topk(k, dim=1, largest=False).indices  # (n, k)
    dst = torch.arange(n).repeat_interleave(k)
    src = nbr.reshape(-1)
    return src, dst


def seeded_parameters(model, seed: int) -> None:
    """Fill every parameter (not buffer) of ``model`` from one generator, in sorted-name
    order: U(-1, 1) / sqrt(last dim).  The B200 modules have the same parameter names and
    shapes, so the same call reproduces the weights without storing them."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(model.named_parameters()):
            scale = 1.0 / max(1, p.shape[-1]) ** 0.5 if p.dim() else 0.1
            p.copy_((torch.rand(p.shape, generator=g, dtype=torch.float64) * 2 - 1).to(p.dtype) * scale)


def knn_within(coords: torch.Tensor, batch: torch.Tensor, k: int):
    """k nearest neighbours inside each graph of a batch, src -> dst, grouped by dst."""
    return knn_graph(coords, k, batch)


def make_model_config4(fe) -> dict:
    """benchmark config 4 at reduced size: EquivariantTransformer in Repr([0,1],32), hidden
    Repr([0,1,2,3],128), 8 heads, 16-NN within each graph, coordinates N(0, 2^2), seed 3.
    Out Repr([0], 8) instead of Repr([0], 1): the reference rejects 8 heads on out mult 1
    (attention.py:233-236).  3 layers (in -> hidden, hidden -> hidden, hidden -> out) on
    4 graphs of 50 nodes; weights from seeded_parameters(model, 3)."""
    n_graphs, npg, k = 4, 50, 16
    g = torch.Generator().manual_seed(3)
    coords = torch.randn(n_graphs * npg, 3, generator=g) * 2.0
    batch = torch.arange(n_graphs).repeat_interleave(npg)
    src, dst = knn_within(coords, batch, k)
    x = torch.randn(n_graphs * npg, 32, 4, generator=g)
    rin, rh, rout = fe.Repr([0, 1], mult=32), fe.Repr([0, 1, 2, 3], mult=128), fe.Repr([0], mult=8)
    model = fe.EquivariantTransformer(rin, rh, rout, num_layers=3, num_heads=8, max_dist=10.0).eval()
    seeded_parameters(model, 3)
    graph = fe.Graph(src=src, dst=dst, num_nodes=len(coords))
    caps = []
    hooks = [lay.register_forward_hook(lambda mod, inp, outp: caps.append(outp)) for lay in model.layers]
    with torch.no_grad():
        y = model(coords, x, graph)
    for h in hooks:
        h.remove()
    return {"coords": coords, "src": src, "dst": dst, "x": x, "output": y, "first_layer_output": caps[0],
            "param_seed": 3, "num_layers": 3, "num_heads": 8}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=["all", "model4"], default="all",
                    help="model4: only the config-4 model fixture (model_config4.pt)")
    ap.add_argument("--ref", default=os.environ.get("FEQ_REFERENCE_ROOT")
                    or os.path.join(os.path.dirname(ROOT), "reference"))
    args = ap.parse_args()
    fe, orc = import_reference(args.ref)
    if args.only == "model4":
        torch.save(make_model_config4(fe), os.path.join(HERE, "model_config4.pt"))
        print("model_config4.pt", os.path.getsize(os.path.join(HERE, "model_config4.pt")))
        return 0
    from flash_eq.layers.linear import EquivariantEdgewiseLinear
    from flash_eq.representations.wigner import _build_m_order_permutation

    out: dict = {}

    # ---- 1. representation bookkeeping (integer, exact) --------------------
    lvals_sets = [[0], [1], [2], [0, 1], [0, 1, 2], [1, 2], [0, 2], [1, 2, 3], [0, 0], [1, 1],
                  [0, 1, 1], [1, 2, 2], [0, 1, 2, 3], [0, 1, 2, 3, 4], [0, 1, 2, 3, 4, 5], [3, 0, 2],
                  [2, 2, 0, 1], [6], [0, 1, 2, 3, 4, 5, 6]]
    book = {"perm": {}, "dim": {}, "cumdims": {}, "mvals": {}, "find_scalar": {}, "nreps": {},
            "block_sizes": {}, "l_indices": {}}
    from flash_eq.cuda.block_diagonal import _compute_block_sizes
    for lv in lvals_sets:
        key = ",".join(map(str, lv))
        r = fe.Repr(lv, mult=3)
        book["perm"][key] = _build_m_order_permutation(r.lvals).tolist()
        book["dim"][key] = r.dim()
        book["cumdims"][key] = r.cumdims().tolist()
        book["mvals"][key] = r.mvals().tolist()
        book["find_scalar"][key] = list(r.find_scalar())
        book["l_indices"][key] = r.l_indices().tolist()
    for a in lvals_sets:
        for b in lvals_sets[:12]:
            key = ",".join(map(str, a)) + "|" + ",".join(map(str, b))
            pr = fe.ProductRepr(fe.Repr(a), fe.Repr(b))
            book["nreps"][key] = pr.nreps()
            book["block_sizes"][key] = list(_compute_block_sizes(torch.tensor(a, dtype=torch.int32),
                                                                 torch.tensor(b, dtype=torch.int32)))
    with open(os.path.join(HERE, "bookkeeping.json"), "w") as fh:
        json.dump(book, fh, indent=0, sort_keys=True)

    # ---- 2. Wigner-D basis (reference matrix_exp path) ---------------------
    g = torch.Generator().manual_seed(11)
    dirs = torch.randn(40, 3, generator=g)
    special = torch.tensor([[0.0, 0.0, 0.0], [0.0, 0.0, 1.0], [0.0, 0.0, -1.0], [1.0, 0.0, 0.0],
                            [0.0, 1.0, 0.0], [-1.0, 0.0, 0.0], [1e-10, 1e-10, 1e-10], [1e-20, 0.0, 0.0],
                            [1e-4, 0.0, -1.0], [0.0, 1e-4, 1.0], [3.0, 4.0, 0.0], [1e-3, -1e-3, -1.0]])
    dirs = torch.cat([dirs, special, dirs[:4] * 1e3])
    basis_fx = {"directions": dirs}
    for lv in ([0, 1, 2], [0, 1, 2, 3, 4], [0, 1, 1], [1, 2, 2], [0, 2], [5], [0, 1, 2, 3, 4, 5, 6], [3, 1]):
        (M,) = fe.WignerDBasis([fe.Repr(lv)])(dirs)
        basis_fx["P_" + ",".join(map(str, lv))] = M.clone()
    # rot() for general axes (used by equivariance tests): axis/angle pairs
    ax = torch.randn(8, 3, generator=g)
    ax = ax / ax.norm(dim=-1, keepdim=True)
    ang = torch.rand(8, generator=g) * 3.14159
    basis_fx["rot_axis"], basis_fx["rot_angle"] = ax, ang
    basis_fx["rot_0,1,2,3"] = fe.WignerD(fe.Repr([0, 1, 2, 3])).rot(ax, ang)
    basis_fx["rot_cart_1"] = fe.WignerD(fe.Repr([1])).rot(ax, ang, cartesian=True)
    basis_fx["rot_to_ez_0,1,2"] = fe.WignerD(fe.Repr([0, 1, 2])).rot_to_ez(dirs)
    torch.save(basis_fx, os.path.join(HERE, "basis.pt"))

    # ---- 3. radial table ---------------------------------------------------
    rad = {}
    for name, kw in (("lin", dict(num_bins=20, out_mult=4, in_mult=3, weight_dim=19, rank=4, hidden_dim=16,
                                  min_val=0.0, max_val=10.0, log=False)),
                     ("log", dict(num_bins=16, out_mult=2, in_mult=5, weight_dim=7, rank=2, hidden_dim=8,
                                  min_val=0.5, max_val=8.0, log=True))):
        torch.manual_seed(5)
        net = fe.SeparableRadialNet(**kw)
        rad[name] = {"kwargs": kw, "state": net.state_dict(), "table": net().detach(),
                     "binning_params": list(net.binning_params())}
        vals = torch.tensor([-1.0, 0.0, 0.3, 0.5, 1.0, 2.5, 7.9, 8.0, 9.99, 10.0, 12.0])
        rad[name]["bin_indices_in"] = vals
        rad[name]["bin_indices_out"] = [x.clone() for x in net.bin_indices(vals)]
    torch.save(rad, os.path.join(HERE, "radial.pt"))

    # ---- 4. edgewise linear (reference layer, oracle kernel) ---------------
    cases = [([0], [0]), ([1], [1]), ([0, 1, 2], [0, 1, 2]), ([1, 2], [1, 2]), ([0, 2], [0, 2]),
             ([1, 2, 3], [1, 2, 3]), ([0], [0, 1]), ([0, 1], [0, 1, 2]), ([1, 2], [0, 1, 2]),
             ([0, 1, 2], [1, 2]), ([2], [0, 1, 2]), ([0, 1], [2]), ([0, 0], [0, 0]), ([0, 1, 1], [0, 1, 2]),
             ([1, 2, 2], [0, 1]), ([0, 1, 2, 3, 4], [0, 1, 2, 3, 4]), ([0, 1, 2, 3, 4, 5], [0, 1, 2, 3, 4, 5])]
    ew = []
    for ci, (lin, lout) in enumerate(cases):
        torch.manual_seed(100 + ci)
        mult_in, mult_out = (3, 5) if ci % 2 else (4, 4)
        rin, rout = fe.Repr(lin, mult=mult_in), fe.Repr(lout, mult=mult_out)
        log_bins = ci % 5 == 4
        layer = EquivariantEdgewiseLinear(rin, rout, num_bins=50, min_dist=0.2 if log_bins else 0.0,
                                          max_dist=6.0, log_bins=log_bins)
        basis = fe.WignerDBasis([rin, rout])
        E = 60
        feats = torch.randn(E, mult_in, rin.dim())
        dirs_e = torch.randn(E, 3)
        dist = torch.rand(E) * 6.5  # includes a few beyond max_dist (extrapolation)
        dist[:3] = torch.tensor([0.0, 6.0, 7.0])
        P, Q = basis(dirs_e)
        with torch.no_grad():
            y = layer(P, Q, feats, dist)
        ew.append({"lvals_in": lin, "lvals_out": lout, "mult_in": mult_in, "mult_out": mult_out,
                   "num_bins": 50, "min_dist": layer.radial_weights.min_val, "max_dist": 6.0,
                   "log_bins": log_bins, "state": layer.state_dict(), "features": feats,
                   "directions": dirs_e, "distances": dist, "output": y})
    torch.save(ew, os.path.join(HERE, "edgewise.pt"))

    # config-1 shaped (scaled down): Repr([0,1,2],32), kNN graph, dst - src directions
    torch.manual_seed(0)
    g0 = torch.Generator().manual_seed(0)
    N, k = 64, 16
    coords = torch.randn(N, 3, generator=g0) * 3.0
    src, dst = knn_graph(coords, k)
    x = torch.randn(N, 32, 9, generator=g0)
    rr = fe.Repr([0, 1, 2], mult=32)
    torch.manual_seed(0)
    layer = EquivariantEdgewiseLinear(rr, rr, num_bins=100, min_dist=0.0, max_dist=10.0)
    vec = coords[dst] - coords[src]
    dist = vec.norm(dim=-1)
    P, Q = fe.WignerDBasis([rr, rr])(vec)
    with torch.no_grad():
        y = layer(P, Q, x[src], dist)
    torch.save({"coords": coords, "src": src, "dst": dst, "x": x, "state": layer.state_dict(),
                "output": y, "distances": dist}, os.path.join(HERE, "edgewise_cfg1_small.pt"))

    # ---- 5. attention + pooling --------------------------------------------
    torch.manual_seed(7)
    gq = torch.Generator().manual_seed(7)
    N, E, H = 12, 70, 4
    src = torch.randint(0, N, (E,), generator=gq)
    dst = torch.randint(0, N - 2, (E,), generator=gq)     # nodes N-2, N-1 have no in-edges
    Qe, Ke = torch.randn(E, H, 10, generator=gq), torch.randn(E, H, 10, generator=gq)
    V = torch.randn(E, 8, 9, generator=gq)
    dist = torch.rand(E, generator=gq) * 5
    graph = fe.Graph(src=src, dst=dst, num_nodes=N)
    att = {"src": src, "dst": dst, "N": N, "Q": Qe, "K": Ke, "V": V, "distances": dist}
    for decay in (None, 3.0):
        m = fe.EquivariantEdgeAttention(num_heads=H, qk_dim=10, distance_decay_scale=decay)
        with torch.no_grad():
            att[f"out_decay{decay}"] = m(Qe, Ke, V, graph, dist)
            att[f"log_scale_decay{decay}"] = m.log_scale.detach().clone()
    m1 = fe.EquivariantEdgeAttention(num_heads=1, qk_dim=40)
    with torch.no_grad():
        att["out_h1"] = m1(Qe.reshape(E, 1, 40), Ke.reshape(E, 1, 40), V, graph)
    for red in ("sum", "mean", "max"):
        att["pool_" + red] = fe.GraphPooling(red)(V, graph)
    # full EquivariantAttention (reference layer, oracle kernel)
    rin, rout = fe.Repr([0, 1, 2], mult=8), fe.Repr([0, 1], mult=8)
    torch.manual_seed(8)
    ea = fe.EquivariantAttention(rin, rout, num_heads=4, num_bins=30, distance_decay_scale=4.0)
    xn = torch.randn(N, 8, 9, generator=gq)
    dirs_e = torch.randn(E, 3, generator=gq)
    P, Qb = fe.WignerDBasis([rin, rout])(dirs_e)
    edge_add = torch.randn(E, 8, 9, generator=gq)
    with torch.no_grad():
        att["ea_out"] = ea(P, Qb, xn, dist, graph)
        att["ea_out_edgefeat"] = ea(P, Qb, xn, dist, graph, edge_features=edge_add)
    att.update({"ea_state": ea.state_dict(), "ea_x": xn, "ea_dirs": dirs_e, "ea_edge_add": edge_add})
    torch.save(att, os.path.join(HERE, "attention.pt"))

    # ---- 6. transformer block and full transformer -------------------------
    gb = torch.Generator().manual_seed(2)
    nb_graphs, npg = 4, 10
    coords = torch.randn(nb_graphs * npg, 3, generator=gb) * 1.5
    batch = torch.arange(nb_graphs).repeat_interleave(npg)
    dd = torch.cdist(coords, coords)
    mask = (dd < 3.0) & (batch[:, None] == batch[None, :]) & ~torch.eye(len(coords), dtype=torch.bool)
    dst, src = mask.nonzero(as_tuple=True)
    graph = fe.Graph(src=src, dst=dst, num_nodes=len(coords))
    rr = fe.Repr([0, 1, 2], mult=16)
    blk = {"coords": coords, "src": src, "dst": dst}
    for name, kw in (("std", dict(num_heads=4, max_dist=10.0)),
                     ("ls_none", dict(num_heads=2, max_dist=10.0, layer_scale_init=None,
                                      distance_decay_scale=2.0)),
                     ("change", dict(num_heads=4, max_dist=10.0))):
        torch.manual_seed(21)
        rout = fe.Repr([0, 1], mult=8) if name == "change" else rr
        block = fe.EquivariantTransformerBlock(rr, rout, **kw)
        block.eval()
        x = torch.randn(len(coords), 16, 9, generator=gb)
        vec = coords[src] - coords[dst]
        dist = vec.norm(dim=-1)
        P, Q = fe.WignerDBasis([rr, rout])(vec)
        captured = {}
        hook = block.attn.register_forward_hook(lambda mod, inp, outp: captured.__setitem__("attn", outp))
        with torch.no_grad():
            y = block(P, Q, x, dist, graph)
        hook.remove()
        blk[name] = {"kwargs": kw, "lvals_out": rout.lvals.tolist(), "mult_out": rout.mult,
                     "state": block.state_dict(), "x": x, "output": y, "attn_out": captured["attn"]}
    torch.save(blk, os.path.join(HERE, "block.pt"))

    torch.manual_seed(3)
    # out mult 4, not 1: the reference rejects num_heads that do not divide out_repr.mult
    # (attention.py:233-234), which also rules out benchmark config 4 as written.
    rin, rh, rout = fe.Repr([0, 1], mult=8), fe.Repr([0, 1, 2], mult=16), fe.Repr([0], mult=4)
    model = fe.EquivariantTransformer(rin, rh, rout, num_layers=3, num_heads=4, max_dist=10.0)
    model.eval()
    x = torch.randn(len(coords), 8, 4, generator=gb)
    caps = []
    hooks = [lay.register_forward_hook(lambda mod, inp, outp: caps.append(outp)) for lay in model.layers]
    with torch.no_grad():
        y = model(coords, x, graph)
    for h in hooks:
        h.remove()
    torch.save({"coords": coords, "src": src, "dst": dst, "x": x, "state": model.state_dict(),
                "output": y, "layer_outputs": caps}, os.path.join(HERE, "transformer.pt"))
    torch.save(make_model_config4(fe), os.path.join(HERE, "model_config4.pt"))

    sizes = {f: os.path.getsize(os.path.join(HERE, f)) for f in os.listdir(HERE) if f.endswith((".pt", ".json"))}
    print(json.dumps(sizes, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
