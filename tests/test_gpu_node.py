"""GPU parity of the native node-level kernels (csrc/feq_node.cu) against the reference
formulation of the same modules (the PyTorch path the modules take under autograd,
flash_eq/layers/norm.py:19-249, gating.py:17-76 of the reference), float64 on the CPU.
Tolerance: 1e-5 relative L2 (single-pass float32 reductions over <= 128 channels)."""
from __future__ import annotations

import copy

import pytest
import torch

import flash_eq as fe
from flash_eq.cuda import ops
from conftest import rel_l2
from flash_eq.layers.gating import EquivariantGating
from flash_eq.layers.norm import EquivariantLayerNorm, RepNorm, SeparableEquivariantLayerNorm

pytestmark = pytest.mark.gpu

REPRS = [([0, 1, 2], 64), ([0, 1, 2, 3], 128), ([0, 0, 1, 2], 7), ([1, 2], 16), ([0], 5), ([0, 1], 1)]


def _randomise(m, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.5 + (1.0 if p.dim() <= 2 else 0.0))


def _check(module, x, dev, tol=1e-5):
    ref = copy.deepcopy(module).double()
    with torch.no_grad():
        y = module.to(dev)(x.to(dev))                  # native kernel
        r = ref(x.double())                            # reference formulation, float64, CPU
    assert y.shape == r.shape
    assert torch.isfinite(y).all()
    assert rel_l2(y, r) < tol


@pytest.mark.parametrize("lv,mult", REPRS, ids=[f"{r[0]}x{r[1]}" for r in REPRS])
def test_separable_layernorm(cuda_device, lv, mult):
    r = fe.Repr(lv, mult=mult)
    m = SeparableEquivariantLayerNorm(r)
    _randomise(m, 1)
    x = torch.randn(300, mult, r.dim(), generator=torch.Generator().manual_seed(2)) * 2 + 0.3
    _check(m, x, cuda_device)


@pytest.mark.parametrize("lv,mult", REPRS, ids=[f"{r[0]}x{r[1]}" for r in REPRS])
def test_equivariant_layernorm(cuda_device, lv, mult):
    r = fe.Repr(lv, mult=mult)
    m = EquivariantLayerNorm(r)
    _randomise(m, 3)
    x = torch.randn(2, 150, mult, r.dim(), generator=torch.Generator().manual_seed(4))
    _check(m, x, cuda_device)


@pytest.mark.parametrize("lv,mult", REPRS[:4], ids=[f"{r[0]}x{r[1]}" for r in REPRS[:4]])
def test_rep_norm_and_gating(cuda_device, lv, mult):
    r = fe.Repr(lv, mult=mult)
    x = torch.randn(257, mult, r.dim(), generator=torch.Generator().manual_seed(5))
    _check(RepNorm(r), x, cuda_device)
    g = EquivariantGating(r)
    _randomise(g, 6)
    _check(g, x, cuda_device, tol=2e-5)


def test_native_and_autograd_paths_agree(cuda_device):
    """Under autograd the modules take the PyTorch path; both paths give the same values."""
    r = fe.Repr([0, 1, 2], mult=32)
    blk = fe.EquivariantTransformerBlock(r, r, num_heads=4, layer_scale_init=0.5).to(cuda_device)
    for mod in (blk.norm1, blk.norm2, blk.attn.norm_qk, blk.mlp_act):
        _randomise(mod, 7)
    x = torch.randn(400, 32, 9, device=cuda_device)
    h = torch.randn(400, 64, 9, device=cuda_device)
    for mod, inp in ((blk.norm1, x), (blk.attn.norm_qk, x), (blk.mlp_act, h), (blk.mlp_up, x)):
        with torch.no_grad():
            a = mod(inp)
        b = mod(inp.clone().requires_grad_())
        assert rel_l2(a, b.detach()) < 1e-5, type(mod).__name__


def _linear_reference(m, f):
    """EquivariantLinear.forward as the reference writes it (linear.py:230-268)."""
    b = f.shape[:-2]
    out = (m.weight @ f).view(*b, *m.outdims)
    out = out.gather(dim=-3, index=m.indices.expand(*b, *m.expanddims)).squeeze(-3)
    if m.bias is not None:
        out = out.clone()
        out[..., m.scalar_locs] = m.activation(out[..., m.scalar_locs] + m.bias)
    return out


LINEAR_CASES = [([0, 1, 2], 64, 128, True), ([0, 1, 2], 128, 64, True), ([0, 0, 1, 2], 8, 6, True),
                ([1, 2], 5, 7, False), ([0, 1, 2, 3], 128, 128, True), ([0, 1, 2, 3, 4], 16, 24, True),
                ([3, 0], 3, 70, True)]


@pytest.mark.parametrize("lv,cin,cout,bias", LINEAR_CASES, ids=[f"{c[0]}-{c[1]}-{c[2]}" for c in LINEAR_CASES])
def test_equivariant_linear(cuda_device, lv, cin, cout, bias):
    m = fe.EquivariantLinear(fe.Repr(lv, mult=cin), fe.Repr(lv, mult=cout), bias=bias)
    if m.bias is not None:
        with torch.no_grad():
            m.bias.normal_()
    f = torch.randn(3, 37, cin, fe.Repr(lv, 1).dim(), generator=torch.Generator().manual_seed(8))
    ref = _linear_reference(copy.deepcopy(m).double(), f.double())
    with torch.no_grad():
        y = m.to(cuda_device)(f.to(cuda_device))
    # shapes the tensor-core kernel serves compute in bf16x3 (float32-level, 1e-4 like the
    # edge path); the others go through the float32 library GEMM
    tol = 1e-4 if ops.node_linear_tc_supported(lv, cin, cout) else 1e-5
    assert y.shape == ref.shape and rel_l2(y, ref) < tol
    yg = m(f.to(cuda_device).requires_grad_())       # the autograd formulation
    assert rel_l2(yg.detach(), ref) < 1e-5
