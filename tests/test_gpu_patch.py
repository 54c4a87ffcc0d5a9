"""PatchedConvSE3 (flash_eq.patch) on the B200 kernels against the reference's computation
(flash_eq/patch/_patched_conv.py:71-129): gather the node features by src, bmm(., P),
block_diagonal_cuda with sh_scale = 0 and 500 bins, bmm(., Q^T), optional self-interaction,
sum onto dst -- here evaluated by the CPU oracle.  The README's patch benchmark shapes
(FULL fuse, C = 32, 500 bins, L = 2 / 3) at 4K edges; a synthetic converted table (the
NVIDIA model and its weight conversion are not part of this build).
Tolerance: 1e-4 relative L2 (bf16x3 mix)."""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import feq_oracle as orc
import flash_eq as fe
from conftest import rel_l2
from flash_eq.patch import PatchedConvSE3


class _FakeGraph:
    def __init__(self, src, dst, n):
        self._s, self._d, self._n = src, dst, n

    def edges(self):
        return self._s, self._d

    def num_nodes(self):
        return self._n


def _conv(L, C, pool, self_int, gen):
    degrees = list(range(L + 1))
    conv = SimpleNamespace(pool=pool, fiber_in=SimpleNamespace(degrees=degrees),
                           fiber_out=SimpleNamespace(degrees=degrees), self_interaction=self_int)
    if self_int:
        conv.to_kernel_self = {str(d): torch.randn(C, C, generator=gen) * 0.1 for d in degrees}
    return conv


@pytest.mark.gpu
@pytest.mark.parametrize("L", [2, 3])
@pytest.mark.parametrize("pool,self_int", [(True, False), (False, False), (True, True)])
def test_patched_conv_matches_reference_computation(cuda_device, L, pool, self_int):
    C, nb, E, N = 32, 500, 4096, 300
    gen = torch.Generator().manual_seed(L + 10 * pool + 100 * self_int)
    lv = list(range(L + 1))
    rin = fe.Repr(lv, mult=C)
    pr = fe.ProductRepr(rin, rin)
    table = torch.randn(nb + 1, C, C, pr.nreps(), generator=gen) * 0.05
    node = {str(d): torch.randn(N, C, 2 * d + 1, generator=gen) for d in lv}
    src = torch.randint(0, N, (E,), generator=gen)
    dst = torch.randint(0, N, (E,), generator=gen)
    rel = torch.randn(E, 3, generator=gen) * 3.0
    dist = rel.norm(dim=-1)
    dirs = rel / dist[:, None]
    conv = _conv(L, C, pool, self_int, gen)
    mod = PatchedConvSE3(conv, table.to(cuda_device), pr, rin, rin, nb, 0.0, 10.0)
    if self_int:
        mod.to_kernel_self = {k: v.to(cuda_device) for k, v in conv.to_kernel_self.items()}
    (M,) = fe.WignerDBasis([fe.Repr(lv)])(dirs.to(cuda_device))
    basis = {"_P": M, "_Q": M, "_distances": dist.to(cuda_device)}
    g = _FakeGraph(src.to(cuda_device), dst.to(cuda_device), N)
    with torch.no_grad():
        out = mod({k: v.to(cuda_device) for k, v in node.items()}, {}, g, basis)
    torch.cuda.synchronize()

    # the reference's steps, on the CPU
    feats = torch.cat([node[str(d)][src] for d in lv], dim=-1)
    P = orc.wigner_basis(dirs, lv)
    y = orc.edgewise_fwd(P, P, feats, dist, table, lv, lv, 0.0, 0.0, nb / 10.0, nb, False)
    if self_int:
        off, parts = 0, []
        for d in lv:
            parts.append(y[..., off:off + 2 * d + 1] + conv.to_kernel_self[str(d)] @ node[str(d)][dst])
            off += 2 * d + 1
        y = torch.cat(parts, dim=-1)
    if pool:
        y = orc.pool(y, dst, N, "sum")
    off = 0
    for d in lv:
        assert rel_l2(out[str(d)], y[..., off:off + 2 * d + 1]) < 1e-4, f"degree {d}"
        off += 2 * d + 1


def test_patch_function_explains_what_is_missing():
    """Host-side only (no GPU)."""
    with pytest.raises(NotImplementedError, match="PatchedConvSE3"):
        fe.patch(torch.nn.Linear(2, 2))
