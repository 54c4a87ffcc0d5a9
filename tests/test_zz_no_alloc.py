"""feq_block_diagonal_fwd_noalloc: the block-diagonal radial mix for callers that
cannot allocate device memory (a host framework that owns all allocations, a plugin
given raw pointers but no allocator).  Its scratch is a fixed array inside the
library, so consecutive calls reuse whatever the previous call left there; these
tests check that the results still equal the ordinary entry point's (which takes a
caller-allocated workspace), call after call, and that a problem too large for the
fixed scratch is refused with a clear message instead of running.

Kept in its own file, collected last, so a run that stops at the first failure has
already run every other test.  Runs alone in a fresh process as well.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import _lib, ops

pytestmark = pytest.mark.gpu


def _noalloc(f, table, dist, lin, lout, sh_scale, p1, p2, nb, log_bins):
    lib = _lib.load()
    E, c_in, _ = f.shape
    c_out = table.shape[1]
    out = torch.empty(E, c_out, sum(2 * l + 1 for l in lout), device=f.device)
    ai, ni = _lib.i32_array(lin)
    ao, no = _lib.i32_array(lout)
    rc = lib.feq_block_diagonal_fwd_noalloc(
        ctypes.c_void_p(f.data_ptr()), ctypes.c_void_p(table.data_ptr()), ctypes.c_void_p(dist.data_ptr()), E,
        c_in, c_out, ai, ni, ao, no, sh_scale, p1, p2, nb, int(log_bins), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def _case(seed, lin, lout, mult, E, nb, log_bins, dev):
    g = torch.Generator().manual_seed(seed)
    rin, rout = fe.Repr(lin, mult), fe.Repr(lout, mult)
    table = torch.randn(nb + 1, mult, mult, fe.ProductRepr(rin, rout).nreps(), generator=g).to(dev)
    f = torch.randn(E, mult, rin.dim(), generator=g).to(dev)
    dist = (torch.rand(E, generator=g) * 12 - 1).to(dev)
    lo_d = 0.5 if log_bins else 0.0
    if log_bins:
        p1 = torch.tensor(lo_d).log().item()
        p2 = 1.0 / torch.tensor(10.0 / lo_d).log().item()
    else:
        p1, p2 = 0.0, nb / 10.0
    return f, table, dist, p1, p2


def test_noalloc_matches_workspace_entry_point_call_after_call(cuda_device):
    cases = [  # consecutive calls with different shapes: stale scratch must not matter
        (1, [0, 1, 2], [0, 1, 2], 16, 20000, 64, False),
        (2, [0, 1, 2, 3], [1, 0], 8, 5000, 100, True),
        (1, [0, 1, 2], [0, 1, 2], 16, 20000, 64, False),
    ]
    for seed, lin, lout, mult, E, nb, log_bins in cases:
        f, table, dist, p1, p2 = _case(seed, lin, lout, mult, E, nb, log_bins, cuda_device)
        ref = ops.block_diagonal_fwd(f, table, dist, lin, lout, 0.1, p1, p2, nb, log_bins)
        rc, y = _noalloc(f, table, dist, lin, lout, 0.1, p1, p2, nb, log_bins)
        torch.cuda.synchronize()
        assert rc == 0, _lib.load().feq_last_error()
        assert rel_l2(y, ref) < 1e-4


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    lv, n = _lib.i32_array([0, 1, 2, 3, 4])
    # config-2 sizes: the re-laid radial table alone is ~140 MB > the fixed scratch
    rc = lib.feq_block_diagonal_fwd_noalloc(None, None, None, 640000, 64, 64, lv, n, lv, n, 0.1, 0.0, 10.0, 100,
                                            0, None, None)
    assert rc == 3                                   # FEQ_ERR_WORKSPACE
    msg = lib.feq_last_error().decode()
    assert "scratch" in msg and "bytes" in msg
