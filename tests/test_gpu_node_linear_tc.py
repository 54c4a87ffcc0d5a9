"""GPU parity of the tensor-core EquivariantLinear kernel (feq_node_linear_tc).

EquivariantLinear.forward (flash_eq/layers/linear.py:230-268 of the reference) computes
weight @ f for every irrep at every position and gathers each position's own irrep; the
kernel computes only those products, per irrep on the tcgen05 tensor cores, with the node
rows read once and the output rows written once.  Reference here: that formulation in
float64 on the CPU.  Tolerances (relative L2): 1e-4 for bf16x3 (the float32 bar of the
edge path), 2e-2 for bf16.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import _lib, ops

pytestmark = pytest.mark.gpu

TOL = {"bf16x3": 1e-4, "bf16": 2e-2}
SHAPES = [(1, 64, 64), (1, 64, 128), (1, 128, 64), (2, 64, 64), (2, 64, 128), (2, 128, 64)]


def _reference(weight, bias, f, lv):
    """y[n, co, p] = sum_ci W[irrep(p)][co, ci] f[n, ci, p] (+ bias[co] at l = 0), float64."""
    w = weight.double()
    y = torch.empty(f.shape[0], w.shape[1], f.shape[2], dtype=torch.float64)
    off = 0
    for r, l in enumerate(lv):
        k = 2 * l + 1
        y[:, :, off:off + k] = torch.einsum("oi,nip->nop", w[r], f[:, :, off:off + k].double())
        off += k
    if bias is not None:
        y[:, :, 0] += bias.double().view(-1)
    return y


def _run(dev, f, lv, w, b, mix):
    cout, cin = w.shape[1], w.shape[2]
    lib = _lib.load()
    arr, n = _lib.i32_array(lv)
    mode = _lib.FEQ_MIX[mix]
    wsb = lib.feq_node_linear_tc_workspace_bytes(cin, cout, arr, n, mode)
    assert wsb > 0
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    y = torch.full((f.shape[0], cout, f.shape[2]), float("nan"), device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    fd, wd = f.to(dev).contiguous(), w.to(dev).contiguous()
    bd = None if b is None else b.to(dev).contiguous()
    rc = lib.feq_node_linear_tc(ctypes.c_void_p(fd.data_ptr()), f.shape[0], cin, cout, arr, n,
                                ctypes.c_void_p(wd.data_ptr()), None if bd is None else ctypes.c_void_p(bd.data_ptr()),
                                mode, ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(ws.data_ptr()), wsb,
                                ctypes.c_void_p(status.data_ptr()), ops._stream(dev))
    _lib.check(rc, "feq_node_linear_tc")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return y


@pytest.mark.parametrize("mix", ["bf16x3", "bf16"])
@pytest.mark.parametrize("N", [1, 16, 17, 1000, 7683])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"L{s[0]}_{s[1]}to{s[2]}" for s in SHAPES])
def test_node_linear_tc_matches_reference(cuda_device, shape, N, mix):
    L, cin, cout = shape
    lv = list(range(L + 1))
    d = (L + 1) ** 2
    g = torch.Generator().manual_seed(100 * L + cin + cout + N)
    f = torch.randn(N, cin, d, generator=g)
    w = torch.randn(L + 1, cout, cin, generator=g) / cin ** 0.5
    b = torch.randn(cout, 1, generator=g)
    y = _run(cuda_device, f, lv, w, b, mix)
    ref = _reference(w, b, f, lv)
    assert torch.isfinite(y).all()
    assert rel_l2(y.cpu().double(), ref) < TOL[mix]


@pytest.mark.parametrize("shape", [(2, 64, 128), (2, 128, 64)])
def test_node_linear_tc_without_bias_and_deterministic(cuda_device, shape):
    L, cin, cout = shape
    lv = list(range(L + 1))
    g = torch.Generator().manual_seed(3)
    f = torch.randn(2049, cin, (L + 1) ** 2, generator=g)
    w = torch.randn(L + 1, cout, cin, generator=g)
    a = _run(cuda_device, f, lv, w, None, "bf16x3")
    c = _run(cuda_device, f, lv, w, None, "bf16x3")
    assert torch.equal(a, c)
    assert rel_l2(a.cpu().double(), _reference(w, None, f, lv)) < 1e-4


def test_module_routes_through_tensor_core_kernel(cuda_device):
    """EquivariantLinear (config-3 MLP shapes) under no_grad launches the re-layout of the
    weights and the tensor-core kernel -- two library launches -- and matches the reference."""
    m = fe.EquivariantLinear(fe.Repr([0, 1, 2], 64), fe.Repr([0, 1, 2], 128)).to(cuda_device)
    with torch.no_grad():
        m.bias.normal_()
    f = torch.randn(7680, 64, 9, device=cuda_device)
    lib = _lib.load()
    n0 = lib.feq_launch_count()
    with torch.no_grad():
        y = m(f)
    torch.cuda.synchronize()
    assert lib.feq_launch_count() - n0 == 2
    w = m.weight.detach().cpu().view(3, 128, 64)
    ref = _reference(w, m.bias.detach().cpu(), f.cpu(), [0, 1, 2])
    assert rel_l2(y.cpu().double(), ref) < 1e-4


def test_unsupported_shapes_are_refused(cuda_device):
    lib = _lib.load()
    for lv, cin, cout in (([0, 1, 2, 3], 128, 128), ([1, 2], 64, 64), ([0, 1, 2], 32, 64), ([0, 1, 2], 128, 128)):
        arr, n = _lib.i32_array(lv)
        assert lib.feq_node_linear_tc_workspace_bytes(cin, cout, arr, n, _lib.FEQ_MIX["bf16x3"]) == 0
        assert not ops.node_linear_tc_supported(lv, cin, cout)
