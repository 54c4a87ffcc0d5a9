"""CPU-only checks of the boundary and the host logic (no kernel is launched).

* libflasheq_b200.so loads without a GPU and exports every function that
  include/flasheq_b200.h declares.
* Representation bookkeeping of the drop-in package equals the reference's
  (fixtures from tests/golden/make_golden.py).
* Reference state dicts load into the B200 modules with strict=True.
* Without a GPU the ops fail loudly (CUDANotAvailableError), never fall back.
"""
from __future__ import annotations

import json
import os
import re

import numpy as np
import pytest
import torch

import flash_eq as fe
from conftest import GOLDEN, ROOT, golden
from flash_eq.cuda import _lib

HEADER = os.path.join(ROOT, "include", "flasheq_b200.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b(feq_[a-z0-9_]+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures and header diverge"
    assert lib.feq_abi_version() == _lib.FEQ_ABI_VERSION
    assert lib.feq_status_string(0) == b"ok"


def test_host_side_validation_without_gpu():
    """Layout checks run on the host before anything touches the device."""
    lib = _lib.load()
    big, n = _lib.i32_array([17])
    # l = 17 exceeds the reference limit (MAX_LVALS = 17 -> l <= 16): unsupported, not a crash
    rc = lib.feq_wigner_basis(None, 10, big, n, 0, None, None)
    assert rc == 2
    neg, n2 = _lib.i32_array([-1])
    assert lib.feq_wigner_basis(None, 10, neg, n2, 0, None, None) == 1
    ok, n3 = _lib.i32_array([0, 1, 2])
    assert lib.feq_wigner_basis(None, 0, ok, n3, 0, None, None) == 0       # empty is fine
    assert lib.feq_wigner_basis(None, 5, ok, n3, 7, None, None) == 1       # bad layout id


def test_repr_bookkeeping_matches_reference():
    with open(os.path.join(GOLDEN, "bookkeeping.json")) as fh:
        book = json.load(fh)
    from flash_eq.representations.wigner import _build_m_order_permutation
    for key in book["perm"]:
        lv = [int(x) for x in key.split(",")]
        r = fe.Repr(lv, mult=3)
        assert _build_m_order_permutation(r.lvals).tolist() == book["perm"][key]
        assert r.dim() == book["dim"][key]
        assert r.cumdims().tolist() == book["cumdims"][key]
        assert r.mvals().tolist() == book["mvals"][key]
        assert list(r.find_scalar()) == book["find_scalar"][key]
        assert r.l_indices().tolist() == book["l_indices"][key]
    from flash_eq.cuda.block_diagonal import _compute_block_sizes
    for key, nreps in book["nreps"].items():
        a, b = ([int(x) for x in s.split(",")] for s in key.split("|"))
        assert fe.ProductRepr(fe.Repr(a), fe.Repr(b)).nreps() == nreps
        assert list(_compute_block_sizes(a, b)) == book["block_sizes"][key]


def test_generators_match_reference_convention():
    import feq_oracle as orc
    for l in range(0, 9):
        ours = fe.Irrep(l)._generators().numpy()
        ref = orc.real_generators(l)
        assert np.abs(ours - ref).max() < 1e-6, l


def test_closed_form_tables_reproduce_matrix_exp():
    """The build-time tables (gen_wigner_tables.py) give the reference basis."""
    import importlib.util
    import feq_oracle as orc
    spec = importlib.util.spec_from_file_location(
        "gen_wigner_tables", os.path.join(ROOT, "flash-eq_b200", "csrc", "gen_wigner_tables.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    g = torch.Generator().manual_seed(1)
    dirs = torch.randn(30, 3, generator=g, dtype=torch.float64)
    for l in (1, 2, 4, 7):
        t = gen.tables_for(l)
        gens = torch.from_numpy(orc.real_generators(l, np.float64))
        for v in dirs:
            d = v / v.norm()
            n = torch.hypot(d[0], d[1])
            th = torch.arccos(d[2])
            c, s = (-d[1] / n).item(), (d[0] / n).item()
            coef = [1.0]
            for m in range(1, l + 1):
                coef += [np.cos(m * th.item()), np.sin(m * th.item())]
            M = t @ np.array(coef)
            R = np.zeros((2 * l + 1, 2 * l + 1))
            R[l, l] = 1.0
            ph = np.arctan2(s, c)
            for m in range(1, l + 1):
                R[l - m, l - m] = R[l + m, l + m] = np.cos(m * ph)
                R[l - m, l + m], R[l + m, l - m] = np.sin(m * ph), -np.sin(m * ph)
            D = R @ M @ R.T
            ref = torch.linalg.matrix_exp(th * (c * gens[0] + s * gens[1])).numpy()
            assert np.abs(D - ref).max() < 1e-9, l


def _load_strict(module, state):
    missing, unexpected = module.load_state_dict(state, strict=True)
    assert not missing and not unexpected


def test_reference_state_dicts_load():
    for case in golden("edgewise.pt"):
        rin = fe.Repr(case["lvals_in"], mult=case["mult_in"])
        rout = fe.Repr(case["lvals_out"], mult=case["mult_out"])
        layer = fe.EquivariantEdgewiseLinear(rin, rout, num_bins=case["num_bins"], min_dist=case["min_dist"],
                                             max_dist=case["max_dist"], log_bins=case["log_bins"])
        _load_strict(layer, case["state"])
    att = golden("attention.pt")
    ea = fe.EquivariantAttention(fe.Repr([0, 1, 2], 8), fe.Repr([0, 1], 8), num_heads=4, num_bins=30,
                                 distance_decay_scale=4.0)
    _load_strict(ea, att["ea_state"])
    blk = golden("block.pt")
    rr = fe.Repr([0, 1, 2], mult=16)
    for name in ("std", "ls_none", "change"):
        rout = fe.Repr(blk[name]["lvals_out"], mult=blk[name]["mult_out"])
        _load_strict(fe.EquivariantTransformerBlock(rr, rout, **blk[name]["kwargs"]), blk[name]["state"])
    tr = golden("transformer.pt")
    model = fe.EquivariantTransformer(fe.Repr([0, 1], 8), fe.Repr([0, 1, 2], 16), fe.Repr([0], 4),
                                      num_layers=3, num_heads=4, max_dist=10.0)
    _load_strict(model, tr["state"])


def test_radial_table_cpu_matches_reference():
    """On the CPU SeparableRadialNet runs its PyTorch modules (the native features are a
    GPU path): identical to the reference table."""
    rad = golden("radial.pt")
    for name, d in rad.items():
        net = fe.SeparableRadialNet(**d["kwargs"])
        _load_strict(net, d["state"])
        with torch.no_grad():
            assert torch.allclose(net(), d["table"], atol=1e-6, rtol=1e-5), name
        assert np.allclose(net.binning_params(), d["binning_params"], rtol=1e-7)
        lo, t = net.bin_indices(d["bin_indices_in"])
        assert torch.equal(lo, d["bin_indices_out"][0]) and torch.allclose(t, d["bin_indices_out"][1])


def test_reference_errors_preserved():
    with pytest.raises(ValueError):
        fe.EquivariantAttention(fe.Repr([0, 1], 8), fe.Repr([0], 1), num_heads=8)   # benchmark config 4 as written
    with pytest.raises(ValueError):
        fe.Graph(src=torch.zeros(3, dtype=torch.long), dst=torch.zeros(2, dtype=torch.long), num_nodes=3)
    with pytest.raises(ValueError):
        fe.Repr([])
    with pytest.raises(ValueError):
        fe.EquivariantLinear(fe.Repr([0, 1]), fe.Repr([0, 2]))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_gpu_fails_loudly():
    r = fe.Repr([0, 1], mult=2)
    with pytest.raises(fe.CUDANotAvailableError):
        fe.WignerDBasis([r])(torch.randn(4, 3))
    layer = fe.EquivariantEdgewiseLinear(r, r)
    P = torch.zeros(4, 4, 4)
    with pytest.raises(fe.CUDANotAvailableError):
        layer(P, P, torch.randn(4, 2, 4), torch.rand(4))
