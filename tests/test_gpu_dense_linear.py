"""GPU parity of the tensor-core dense linear (feq_dense_linear_tc), which runs the dense
nn.Linear of EquivariantGating (flash_eq/layers/gating.py:17-76 of the reference: the
(C * n_irreps)^2 mix of the irrep norms) -- y = x w^T + b -- against the same product in
float64 on the CPU.  Tolerances (relative L2): 1e-4 for bf16x3 (the float32 bar of the
edge path), 2e-2 for bf16.
"""
from __future__ import annotations

import copy

import pytest
import torch

import flash_eq as fe
from conftest import rel_l2
from flash_eq.cuda import _lib, ops

pytestmark = pytest.mark.gpu

SHAPES = [(384, 384), (128, 64), (256, 512), (512, 192), (128, 128)]


@pytest.mark.parametrize("mix,tol", [("bf16x3", 1e-4), ("bf16", 2e-2)])
@pytest.mark.parametrize("n", [1, 63, 64, 65, 7680, 30001])
@pytest.mark.parametrize("m,k", SHAPES)
def test_dense_linear_matches_reference(cuda_device, m, k, n, mix, tol):
    g = torch.Generator().manual_seed(m + 7 * k + n)
    x = torch.randn(n, k, generator=g)
    w = torch.randn(m, k, generator=g) / k ** 0.5
    b = torch.randn(m, generator=g)
    y = ops.dense_linear(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), mix=mix)
    torch.cuda.synchronize()
    ref = x.double() @ w.double().t() + b.double()
    assert y.shape == (n, m) and torch.isfinite(y).all()
    assert rel_l2(y.cpu().double(), ref) < tol


def test_dense_linear_without_bias_is_deterministic(cuda_device):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5000, 384, generator=g).to(cuda_device)
    w = torch.randn(384, 384, generator=g).to(cuda_device)
    a = ops.dense_linear(x, w)
    c = ops.dense_linear(x, w)
    assert torch.equal(a, c)
    assert rel_l2(a.cpu().double(), x.cpu().double() @ w.cpu().double().t()) < 1e-4


def test_gating_uses_the_tensor_core_linear(cuda_device):
    """EquivariantGating at the config-3 hidden representation (128 channels x 3 irreps: a
    384 x 384 linear) launches the norms, the weight re-layout, the dense kernel and the gate,
    and matches the reference formulation (sigmoid of Linear(norms) broadcast per irrep)."""
    r = fe.Repr([0, 1, 2], 128)
    gate = fe.EquivariantGating(r).to(cuda_device)
    x = torch.randn(7680, 128, 9, device=cuda_device)
    lib = _lib.load()
    n0 = lib.feq_launch_count()
    with torch.no_grad():
        y = gate(x)
    torch.cuda.synchronize()
    assert lib.feq_launch_count() - n0 == 4
    ref = copy.deepcopy(gate).cpu().double()(x.cpu().double())     # the reference formulation on the CPU
    assert rel_l2(y.cpu().double(), ref) < 1e-4


def test_unsupported_sizes_are_refused(cuda_device):
    for m, k in ((100, 64), (128, 32), (640, 64), (128, 576)):
        assert not ops.dense_linear_tc_supported(m, k)
