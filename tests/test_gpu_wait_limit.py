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


def _short_limit_then_recover(run, check, must_time_out=True):
    """run(status) with a 1 ns pipeline-wait limit must come back (no hang, no fault) with
    status 2 -- or 0 when must_time_out is False: a kernel whose waits are all short may see
    each phase complete before it first looks at the timer (every 8 polls) -- and with the
    default limit give a result that check() accepts."""
    lib = _lib.load()
    dev = torch.device("cuda:0")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    prev = lib.feq_set_wait_limit_ns(1)
    try:
        run(status)
        torch.cuda.synchronize()
    finally:
        lib.feq_set_wait_limit_ns(prev)
    if must_time_out:
        assert int(status.item()) == 2, "a 1 ns wait limit should have timed out at least one wait"
    else:
        assert int(status.item()) in (0, 2)
    status.zero_()
    out = run(status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    check(out)


@pytest.mark.gpu
def test_node_linear_kernel_short_wait_limit(cuda_device):
    """The tensor-core EquivariantLinear (feq_node_linear_tc): weight copies and MMAs drained
    before the kernel frees its tensor memory."""
    import ctypes
    g = torch.Generator().manual_seed(2)
    N, cin, cout, lv = 50000, 64, 128, [0, 1, 2]
    f = torch.randn(N, cin, 9, generator=g).to(cuda_device)
    w = torch.randn(3, cout, cin, generator=g).to(cuda_device)
    lib = _lib.load()
    arr, n = _lib.i32_array(lv)
    wsb = lib.feq_node_linear_tc_workspace_bytes(cin, cout, arr, n, _lib.FEQ_MIX["bf16x3"])
    ws = torch.empty(wsb, dtype=torch.uint8, device=cuda_device)

    def run(status):
        y = torch.empty(N, cout, 9, device=cuda_device)
        rc = lib.feq_node_linear_tc(ctypes.c_void_p(f.data_ptr()), N, cin, cout, arr, n, ctypes.c_void_p(w.data_ptr()),
                                    None, _lib.FEQ_MIX["bf16x3"], ctypes.c_void_p(y.data_ptr()),
                                    ctypes.c_void_p(ws.data_ptr()), wsb, ctypes.c_void_p(status.data_ptr()),
                                    ops._stream(cuda_device))
        _lib.check(rc, "feq_node_linear_tc")
        return y

    def check(y):
        fd, wd = f.double().cpu(), w.double().cpu()
        ref = torch.empty(N, cout, 9, dtype=torch.float64)
        for r, (a, b) in enumerate(((0, 1), (1, 4), (4, 9))):
            ref[:, :, a:b] = torch.einsum("oi,nip->nop", wd[r], fd[:, :, a:b])
        assert rel_l2(y.cpu().double(), ref) < 1e-4

    # one MMA group and one weight copy per CTA to wait for, each shorter than the polls
    # before the first look at the timer: the limit may not be reached
    _short_limit_then_recover(run, check, must_time_out=False)


@pytest.mark.gpu
def test_dense_linear_kernel_short_wait_limit(cuda_device):
    """The tensor-core dense linear (feq_dense_linear_tc): producer, MMA and converter warps
    leave together, copies and MMAs drained."""
    import ctypes
    g = torch.Generator().manual_seed(4)
    n, m, k = 60000, 384, 384
    x = torch.randn(n, k, generator=g).to(cuda_device)
    w = torch.randn(m, k, generator=g).to(cuda_device)
    lib = _lib.load()
    wsb = lib.feq_dense_linear_tc_workspace_bytes(m, k, _lib.FEQ_MIX["bf16x3"])
    ws = torch.empty(wsb, dtype=torch.uint8, device=cuda_device)

    def run(status):
        y = torch.empty(n, m, device=cuda_device)
        rc = lib.feq_dense_linear_tc(ctypes.c_void_p(x.data_ptr()), n, m, k, ctypes.c_void_p(w.data_ptr()), None,
                                     _lib.FEQ_MIX["bf16x3"], ctypes.c_void_p(y.data_ptr()),
                                     ctypes.c_void_p(ws.data_ptr()), wsb, ctypes.c_void_p(status.data_ptr()),
                                     ops._stream(cuda_device))
        _lib.check(rc, "feq_dense_linear_tc")
        return y

    def check(y):
        assert rel_l2(y.cpu().double(), x.cpu().double() @ w.cpu().double().t()) < 1e-4

    _short_limit_then_recover(run, check)


@pytest.mark.gpu
def test_attention_pooling_ring_short_wait_limit(cuda_device):
    """The ring attention pooling kernel: each warp waits for its copies in flight and leaves."""
    g = torch.Generator().manual_seed(6)
    N, E, C, d, H = 20000, 400000, 64, 9, 8
    src = torch.randint(0, N, (E,), generator=g).to(cuda_device)
    dst = torch.randint(0, N, (E,), generator=g).to(cuda_device)
    qk = torch.randn(N, 2 * C, d, generator=g).to(cuda_device)
    V = torch.randn(E, C, d, generator=g).to(cuda_device)
    perm, offsets, _ = ops.edge_sort(dst, N)

    def run(status):
        return ops.attn_pool(qk, V, src, None, perm, offsets, N, H, 0.3, None, "sum", status=status)

    def check(out):
        ref = ops.attn_pool(qk, V, src, None, perm, offsets, N, H, 0.3, None, "sum")
        assert torch.equal(out, ref)                  # deterministic: bitwise the same result

    # the rows are copied four edges ahead of their use, so a wait rarely outlasts the polls
    # before the first look at the timer: the limit may not be reached
    _short_limit_then_recover(run, check, must_time_out=False)
