"""Pin the CPU oracle before trusting it (no GPU needed).

The oracle (``oracle/feq_oracle.py`` + ``oracle/block_diagonal_ref.c``) is
checked against fixtures produced by importing the reference itself
(``tests/golden/make_golden.py``) and against the reference's own property tests
(equivariance, tests/test_equivariance.py:18-99; self-loop suppression,
tests/test_self_loops.py:42-66; pooling known answers,
tests/test_layers.py:470-536; softmax normalisation, tests/test_attention.py:77-107).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

import feq_oracle as orc
from conftest import GOLDEN, check_equivariance, golden


def _book():
    with open(os.path.join(GOLDEN, "bookkeeping.json")) as fh:
        return json.load(fh)


def _lv(key):
    return [int(x) for x in key.split(",")]


def test_m_first_perm_matches_reference():
    book = _book()
    for key, perm in book["perm"].items():
        assert orc.m_first_perm(_lv(key)).tolist() == perm, key


def test_weight_dim_and_block_sizes_match_reference():
    book = _book()
    for key, nreps in book["nreps"].items():
        a, b = key.split("|")
        la, lb = _lv(a), _lv(b)
        assert orc.weight_dim(la, lb) == nreps, key
        mmax, params = orc.block_layout(la, lb)
        # w_off of the last non-empty block + its size == Wdim (block_diagonal.cu:1253-1258)
        total = 0
        max_in = max_out = 0
        for m, n_in, n_out, in_off, out_off, w_off in params.tolist():
            if n_in and n_out:
                mult = 1 if m == 0 else 2
                assert w_off == total
                total += mult * n_in * n_out
                max_in, max_out = max(max_in, mult * n_in), max(max_out, mult * n_out)
        assert total == nreps, key
        assert [max_in, max_out] == book["block_sizes"][key], key


def test_wigner_basis_matches_reference():
    fx = golden("basis.pt")
    dirs = fx["directions"]
    for key, P in fx.items():
        if not key.startswith("P_"):
            continue
        lv = _lv(key[2:])
        ours = orc.wigner_basis(dirs, lv)
        assert torch.allclose(ours, P, atol=1e-5, rtol=0), (key, (ours - P).abs().max().item())


def test_rot_matches_reference():
    fx = golden("basis.pt")
    ours = orc.rot(fx["rot_axis"], fx["rot_angle"], [0, 1, 2, 3])
    assert torch.allclose(ours, fx["rot_0,1,2,3"], atol=1e-5, rtol=0)


def test_radial_table_matches_reference():
    fx = golden("radial.pt")
    for name, d in fx.items():
        kw = d["kwargs"]
        tab = orc.radial_table(d["state"], kw["num_bins"], kw["min_val"], kw["max_val"], kw["log"],
                               kw["rank"], kw["weight_dim"])
        ref = d["table"].double()
        assert (tab - ref).abs().max().item() <= 1e-5 * max(1.0, ref.abs().max().item()), name
        p1, p2 = orc.binning_params(kw["num_bins"], kw["min_val"], kw["max_val"], kw["log"])
        assert np.allclose([p1, p2], d["binning_params"], rtol=1e-7, atol=0), name


def test_binning_index_matches_module_bin_indices():
    """The kernel's bin index equals SeparableRadialNet.bin_indices' (radial.py:285-296).
    In linear mode t agrees wherever the module's clamp to [0, 1] is inactive; in log
    mode the kernel interpolates linearly in distance between the exp'd edges
    (block_diagonal.cu:97-106) while the module interpolates in log space, so only
    the range [0, 1] is shared."""
    fx = golden("radial.pt")
    for name, d in fx.items():
        kw = d["kwargs"]
        p1, p2 = d["binning_params"]
        lo, t = orc.binning(d["bin_indices_in"].numpy(), p1, p2, kw["num_bins"], kw["log"])
        ref_lo, ref_t = d["bin_indices_out"]
        assert lo.tolist() == ref_lo.tolist(), name
        if kw["log"]:
            assert ((t >= 0) & (t <= 1)).all(), name
        else:
            inside = (t >= 0) & (t <= 1)
            assert np.allclose(t[inside], ref_t.numpy()[inside], atol=2e-6), name


def test_binning_linear_unclamped_extrapolation():
    """Linear mode leaves t unclamped (block_diagonal.cu:107-111)."""
    lo, t = orc.binning(np.array([-5.0, 0.0, 5.0, 100.0], np.float32), 0.0, 10.0, 100, False)
    assert lo.tolist() == [0, 0, 50, 99]
    assert t[0] < 0 and t[3] > 1 and abs(t[2]) < 1e-6


def test_edgewise_golden_consistency():
    """Reference layer (with this oracle injected) == oracle chain built from the saved state."""
    for case in golden("edgewise.pt"):
        lin, lout = case["lvals_in"], case["lvals_out"]
        st = case["state"]
        wd = orc.weight_dim(lin, lout)
        tab = orc.radial_table(st, case["num_bins"], case["min_dist"], case["max_dist"], case["log_bins"],
                               4, wd, prefix="radial_weights.").float()
        p1, p2 = orc.binning_params(case["num_bins"], case["min_dist"], case["max_dist"], case["log_bins"])
        P = orc.wigner_basis(case["directions"], lin)
        Q = orc.wigner_basis(case["directions"], lout)
        y = orc.edgewise_fwd(P, Q, case["features"], case["distances"], tab, lin, lout, 0.1, p1, p2,
                             case["num_bins"], case["log_bins"])
        ref = case["output"]
        err = (y - ref).norm() / ref.norm()
        assert err < 1e-5, (lin, lout, err.item())


LVALS_CONFIGS = [([0], [0]), ([1], [1]), ([2], [2]), ([0, 1], [0, 1]), ([0, 1, 2], [0, 1, 2]),
                 ([1, 2], [1, 2]), ([0, 2], [0, 2]), ([1, 2, 3], [1, 2, 3]), ([0], [0, 1]),
                 ([0, 1], [0, 1, 2]), ([1], [0, 1]), ([1, 2], [0, 1, 2]), ([0, 1, 2], [1, 2]),
                 ([2], [0, 1, 2]), ([0, 1], [2]), ([0, 0], [0, 0]), ([1, 1], [1, 1]),
                 ([0, 1, 1], [0, 1, 1]), ([1, 2, 2], [1, 2, 2]), ([0, 1, 1], [0, 1, 2]), ([1, 2, 2], [0, 1])]


def _random_axis_angle(g):
    axis = torch.randn(3, generator=g)
    axis = axis / axis.norm()
    angle = torch.rand(1, generator=g) * 3.14159
    return axis, angle


def _rotations(axis, angle, lvals):
    """Pairing used by the reference's equivariance tests (tests/test_equivariance.py:74-76,
    tests/helpers.py:76-93): features rotate by rot(axis, angle); directions by the
    l=1 block of rot(axis, angle, cartesian=True), i.e. the axis permuted to [z, x, y]."""
    D = orc.rot(axis[None], angle, lvals)[0].double()
    R = orc.rot(axis[[2, 0, 1]][None], angle, [1])[0].double()
    return D, R


@pytest.mark.parametrize("lin,lout", LVALS_CONFIGS)
def test_oracle_equivariance(lin, lout):
    """Reference property D_out f(x, d) = f(D_in x, R d) holds for the oracle chain."""
    g = torch.Generator().manual_seed(42)
    mult, E = 4, 50
    din = sum(2 * l + 1 for l in lin)
    wd = orc.weight_dim(lin, lout)
    table = torch.randn(51, mult, mult, wd, generator=g, dtype=torch.float64)
    f = torch.randn(E, mult, din, generator=g, dtype=torch.float64)
    dirs = torch.randn(E, 3, generator=g, dtype=torch.float64)
    dist = torch.rand(E, generator=g, dtype=torch.float64) * 5
    axis, angle = _random_axis_angle(g)
    D_in, R1 = _rotations(axis, angle, lin)
    D_out, _ = _rotations(axis, angle, lout)
    p1, p2 = 0.0, 50 / 10.0
    def run(ff, dd):
        P = orc.wigner_basis(dd.float(), lin).double()
        Q = orc.wigner_basis(dd.float(), lout).double()
        return orc.edgewise_fwd(P, Q, ff, dist, table, lin, lout, 0.1, p1, p2, 50, False)
    y1 = torch.einsum("ij,ecj->eci", D_out, run(f, dirs))
    y2 = run(torch.einsum("ij,ecj->eci", D_in, f), dirs @ R1.T)
    check_equivariance(y1, y2, rtol=1e-4)


def test_oracle_self_loop_suppresses_higher_l():
    g = torch.Generator().manual_seed(3)
    lv = [0, 1, 2]
    wd = orc.weight_dim(lv, lv)
    table = torch.randn(101, 8, 8, wd, generator=g)
    f = torch.randn(10, 8, 9, generator=g)
    P = orc.wigner_basis(torch.zeros(10, 3), lv)
    y = orc.edgewise_fwd(P, P, f, torch.zeros(10), table, lv, lv, 0.1, 0.0, 10.0, 100, False)
    assert y[..., 1:].abs().max() < 1e-6
    assert y[..., 0].abs().max() > 0


def test_oracle_attention_matches_reference():
    fx = golden("attention.pt")
    dst, N = fx["dst"], fx["N"]
    for decay in (None, 3.0):
        scale = fx[f"log_scale_decay{decay}"].exp()
        ours = orc.edge_attention(fx["Q"], fx["K"], fx["V"], dst, N, scale, 4, fx["distances"], decay)
        assert torch.allclose(ours, fx[f"out_decay{decay}"], atol=1e-6), decay
    for red in ("sum", "mean", "max"):
        assert torch.allclose(orc.pool(fx["V"], dst, N, red), fx["pool_" + red], atol=1e-6), red


def test_oracle_softmax_sums_to_one():
    g = torch.Generator().manual_seed(0)
    dst = torch.randint(0, 20, (100,), generator=g)
    w = orc.segment_softmax(torch.randn(100, 2, generator=g), dst, 20)
    sums = torch.zeros(20, 2).scatter_add_(0, dst.view(-1, 1).expand(-1, 2), w)
    has = torch.zeros(20, dtype=torch.bool)
    has[dst] = True
    assert torch.allclose(sums[has], torch.ones_like(sums[has]), atol=1e-5)


def test_oracle_pooling_known_answers():
    ef = torch.tensor([[[1.0, 2.0]], [[3.0, 4.0]], [[5.0, 6.0]], [[7.0, 8.0]]])
    dst = torch.tensor([0, 0, 1, 1])
    assert torch.equal(orc.pool(ef, dst, 2, "sum"), torch.tensor([[[4.0, 6.0]], [[12.0, 14.0]]]))
    ef = torch.tensor([[[2.0, 4.0]], [[4.0, 8.0]], [[9.0, 3.0]]])
    dst = torch.tensor([0, 0, 1])
    assert torch.equal(orc.pool(ef, dst, 2, "mean"), torch.tensor([[[3.0, 6.0]], [[9.0, 3.0]]]))
    ef = torch.tensor([[[1.0, 5.0]], [[3.0, 2.0]], [[7.0, 8.0]]])
    assert torch.equal(orc.pool(ef, dst, 2, "max"), torch.tensor([[[3.0, 5.0]], [[7.0, 8.0]]]))
