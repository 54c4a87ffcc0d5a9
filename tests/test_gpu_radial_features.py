"""GPU parity of the one-launch radial features (feq_radial_features) that
SeparableRadialNet.radial_features uses on the GPU without autograd, against the module's
PyTorch formulation of radial.py:226-267 (sinusoid x envelope basis, two SiLU layers, head)
in float64 on the CPU.  Tolerance 1e-5 relative L2 (float32 dot products of <= 128 terms)."""
from __future__ import annotations

import copy

import pytest
import torch

from conftest import rel_l2
from flash_eq.layers.radial import SeparableRadialNet

pytestmark = pytest.mark.gpu

CASES = [
    dict(num_bins=100, out_mult=64, in_mult=64, weight_dim=95, rank=4),                    # config 2's layer
    dict(num_bins=100, out_mult=64, in_mult=64, weight_dim=19, rank=4),                    # L <= 2
    dict(num_bins=500, out_mult=32, in_mult=32, weight_dim=7, rank=4, num_freqs=8),
    dict(num_bins=64, out_mult=8, in_mult=8, weight_dim=19, rank=2, hidden_dim=128, min_val=0.5, max_val=6.0,
         log=True),
    dict(num_bins=1, out_mult=4, in_mult=4, weight_dim=3, rank=1, num_freqs=1, hidden_dim=1),
]


def _reference(net: SeparableRadialNet) -> torch.Tensor:
    ref = copy.deepcopy(net).cpu().double()
    with torch.enable_grad():            # the PyTorch path of the module
        f = ref.head(ref.trunk(ref._sinusoidal_basis(ref.bin_edges)))
    return f.detach().view(-1, ref.rank, ref.weight_dim)


@pytest.mark.parametrize("case", CASES, ids=[f"bins{c['num_bins']}_w{c['weight_dim']}_r{c['rank']}" for c in CASES])
def test_radial_features_match_module_formulation(cuda_device, case):
    torch.manual_seed(sum(case[k] for k in ("num_bins", "weight_dim", "rank")))
    net = SeparableRadialNet(**case)
    with torch.no_grad():
        for p in net.parameters():
            p.add_(torch.randn_like(p) * 0.3)
    net = net.to(cuda_device)
    with torch.no_grad():
        assert net._native_features_ok()
        f = net.radial_features()
    torch.cuda.synchronize()
    ref = _reference(net)
    assert f.shape == ref.shape
    assert torch.isfinite(f).all()
    assert rel_l2(f.cpu().double(), ref) < 1e-5


def test_autograd_keeps_the_pytorch_path(cuda_device):
    """With gradients enabled the features come from the nn.Modules, so the radial net
    trains; both paths agree."""
    net = SeparableRadialNet(num_bins=50, out_mult=16, in_mult=16, weight_dim=19).to(cuda_device)
    assert not net._native_features_ok()
    f_grad = net.radial_features()
    f_grad.sum().backward()
    assert net.head.weight.grad is not None
    with torch.no_grad():
        f_native = net.radial_features()
    assert rel_l2(f_native.double(), f_grad.detach().double()) < 1e-5
