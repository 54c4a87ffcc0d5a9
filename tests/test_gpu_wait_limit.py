"""The time-out path of the tensor-core pipelines, made to run out on purpose (no fault).

Every pipeline wait in the tcgen05 kernels (TMA / bulk-copy arrivals, MMA completion,
TMEM hand-over) is bounded; when a wait passes its limit the kernel raises its abort
flag, waits for its own copies and MMAs in flight, frees its tensor memory, returns and
leaves status 2 in the caller's status word.  The limit is a launch parameter
(feq_set_wait_limit_ns), so a test can shrink it to a nanosecond: the ordinary waits for
HBM data then run out.  The call must come back with status 2, the context must stay
usable, and the next call with the default limit must be correct again.
"""
from __future__ import annotations

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import _lib, ops


def _problem(dev, lv, mult, E, seed=3):
    torch.manual_seed(seed)
    r = fe.Repr(lv, mult=mult)
    layer = fe.EquivariantEdgewiseLinear(r, r).to(dev)
    g = torch.Generator().manual_seed(seed + 1)
    f = torch.randn(E, mult, r.dim(), generator=g)
    dirs = torch.randn(E, 3, generator=g)
    dist = torch.rand(E, generator=g) * 10
    rw = layer.radial_weights
    with torch.no_grad():
        table = rw()
    p1, p2 = rw.binning_params()
    return layer, f, dirs, dist, table, p1, p2


def _call(dev, lv, mult, prob, mix, status):
    layer, f, dirs, dist, table, p1, p2 = prob
    rw = layer.radial_weights
    return ops.edgewise_fwd(f.to(dev), dist.to(dev), table, lv, lv, mult, 0.1, p1, p2, rw.num_bins, False,
                            directions=dirs.to(dev), status=status, mix=mix)


@pytest.mark.gpu
@pytest.mark.parametrize("mix", ["bf16x3", "bf16"])
def test_short_wait_limit_returns_status_2_then_recovers(cuda_device, mix):
    lib = _lib.load()
    lv, mult, E = [0, 1, 2, 3, 4], 64, 200000
    prob = _problem(cuda_device, lv, mult, E)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    # 1 ns: any wait that sees the global timer tick at all runs out (the timer's resolution
    # is coarse, so among the many waits of a 200k-edge call some always do)
    prev = lib.feq_set_wait_limit_ns(1)
    try:
        _call(cuda_device, lv, mult, prob, mix, status)
        torch.cuda.synchronize()                        # the kernels returned: no hang, no fault
    finally:
        lib.feq_set_wait_limit_ns(prev)
    assert int(status.item()) == 2, "a 1 ns wait limit should have timed out at least one wait"

    # the context is intact and the default limit gives the right answer again
    status.zero_()
    y = _call(cuda_device, lv, mult, prob, mix, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    layer, f, dirs, dist, table, p1, p2 = prob
    ref = orc.edgewise_fwd(orc.wigner_basis(dirs, lv), orc.wigner_basis(dirs, lv), f, dist, table.cpu(), lv, lv,
                           0.1, p1, p2, layer.radial_weights.num_bins, False)
    assert rel_l2(y, ref) < (1e-4 if mix == "bf16x3" else 2e-2)


def test_wait_limit_setter_round_trips():
    """Host-side only (no GPU): the setter stores the limit and 0 restores the default."""
    lib = _lib.load()
    prev = lib.feq_set_wait_limit_ns(123456)
    try:
        assert lib.feq_set_wait_limit_ns(0) == 123456      # 0 restores the default
        assert lib.feq_set_wait_limit_ns(prev) == 4_000_000_000
    finally:
        lib.feq_set_wait_limit_ns(prev)


@pytest.mark.gpu
@pytest.mark.parametrize("mix", ["bf16x3", "bf16"])
def test_separable_kernel_short_wait_limit(cuda_device, mix):
    """The same for the one-kernel separable edgewise path (feq_edgewise_separable_fwd)."""
    lib = _lib.load()
    lv, mult, E = [0, 1, 2, 3, 4], 64, 200000
    layer, f, dirs, dist, table, p1, p2 = _problem(cuda_device, lv, mult, E, seed=5)
    rw = layer.radial_weights

    def call(status):
        with torch.no_grad():
            return ops.edgewise_separable_fwd(f.to(cuda_device), dist.to(cuda_device), rw.channel_patterns,
                                              rw.radial_features(), lv, lv, 0.1, p1, p2, rw.num_bins, False,
                                              directions=dirs.to(cuda_device), status=status, mix=mix)

    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    prev = lib.feq_set_wait_limit_ns(1)
    try:
        call(status)
        torch.cuda.synchronize()
    finally:
        lib.feq_set_wait_limit_ns(prev)
    assert int(status.item()) == 2
    status.zero_()
    y = call(status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = orc.edgewise_fwd(orc.wigner_basis(dirs, lv), orc.wigner_basis(dirs, lv), f, dist, table.cpu(), lv, lv,
                           0.1, p1, p2, rw.num_bins, False)
    assert rel_l2(y, ref) < (1e-4 if mix == "bf16x3" else 2e-2)
