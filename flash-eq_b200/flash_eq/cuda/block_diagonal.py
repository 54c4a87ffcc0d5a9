"""``block_diagonal_cuda``: the reference's operator boundary, on B200 kernels.

Same signature and contract as flash_eq/cuda/block_diagonal.py:206-274 in
hmblair/flash-eq: features (E, Cin, Din) and output (E, Cout, Dout) in the
m-first basis, radial table (num_bins + 1, Cout, Cin, W), distances (E,).

Differences in mechanism (not in results): no argsort/gather/unsort copies
(edges are grouped by bin inside the native op), no host synchronisation, work
is enqueued on the current stream.  The backward (``_BlockDiagonalFunction``,
block_diagonal.py:100-174 in the reference) runs the native
``feq_block_diagonal_bwd``: grad_features, grad_table and grad_distances,
deterministic (no atomics).  Other native ops of this package are forward only and
raise ``NotImplementedError`` if autograd reaches them.
"""
from __future__ import annotations

import torch

from . import ops
from .ops import CUDANotAvailableError

__all__ = ["block_diagonal_cuda", "CUDANotAvailableError"]


def _compute_block_sizes(lvals_in, lvals_out) -> tuple[int, int]:
    """Max 2x-doubled block sizes (flash_eq/cuda/block_diagonal.py:181-203)."""
    lin = [int(x) for x in (lvals_in.tolist() if torch.is_tensor(lvals_in) else lvals_in)]
    lout = [int(x) for x in (lvals_out.tolist() if torch.is_tensor(lvals_out) else lvals_out)]
    max_in = max_out = 0
    for m in range(max(max(lin), max(lout)) + 1):
        n_in = sum(1 for l in lin if l >= m)
        n_out = sum(1 for l in lout if l >= m)
        if n_in and n_out:
            k = 1 if m == 0 else 2
            max_in, max_out = max(max_in, k * n_in), max(max_out, k * n_out)
    return max_in, max_out


class _ForwardOnly(torch.autograd.Function):
    @staticmethod
    def forward(ctx, fn, *tensors):
        return fn(*tensors)

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError(
            "flash-eq B200: the backward pass of the edge-message kernels is not part of this build "
            "(forward / inference only)."
        )


def forward_only(fn, *tensors):
    """Run ``fn(*tensors)``; if autograd tracks any input, a later backward raises."""
    if torch.is_grad_enabled() and any(t.requires_grad for t in tensors if torch.is_tensor(t)):
        return _ForwardOnly.apply(fn, *tensors)
    return fn(*tensors)


def block_diagonal_cuda(
    features: torch.Tensor,
    radial_table: torch.Tensor,
    distances: torch.Tensor,
    product_repr,
    bin_param1: float,
    bin_param2: float,
    num_bins: int,
    log_bins: bool = False,
    sh_scale: float = 0.1,
    *,
    mix: str = "fp32",
) -> torch.Tensor:
    """out[e] = Lambda(r_e) f[e] in the m-first basis (see module docstring).

    ``mix`` (not a reference argument): "fp32" CUDA-core float32 (default), "bf16x3" or
    "bf16" tensor cores.  The backward always runs on the tensor cores ("bf16x3" unless
    "bf16" is asked for).
    """
    if not torch.cuda.is_available():
        raise CUDANotAvailableError("flash-eq requires a CUDA-capable GPU. No CUDA device was detected.")
    lvals_in = product_repr.rep1.lvals.tolist()
    lvals_out = product_repr.rep2.lvals.tolist()
    num_edges = features.size(0)
    channels_out = radial_table.size(1)
    dim_out = product_repr.rep2.dim()
    if num_edges == 0:
        return torch.zeros(0, channels_out, dim_out, device=features.device, dtype=features.dtype)
    if max(max(lvals_in), max(lvals_out)) >= 17:
        raise RuntimeError("Maximum l-value exceeds supported limit (16).")
    dist = distances.to(features.dtype)
    cfg = (tuple(lvals_in), tuple(lvals_out), float(sh_scale), float(bin_param1), float(bin_param2), int(num_bins),
           bool(log_bins), mix)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (features, radial_table, dist)):
        return _BlockDiagonalFunction.apply(features, radial_table, dist, cfg)
    return ops.block_diagonal_fwd(features.detach(), radial_table.detach(), dist.detach(), lvals_in, lvals_out,
                                  sh_scale, bin_param1, bin_param2, num_bins, log_bins, mix=mix)


class _BlockDiagonalFunction(torch.autograd.Function):
    """Autograd of block_diagonal_cuda (flash_eq/cuda/block_diagonal.py:100-174)."""

    @staticmethod
    def forward(ctx, features, radial_table, dist, cfg):
        lin, lout, sh, p1, p2, nb, log, mix = cfg
        ctx.cfg = cfg
        ctx.save_for_backward(features, radial_table, dist)
        return ops.block_diagonal_fwd(features.detach(), radial_table.detach(), dist.detach(), list(lin), list(lout),
                                      sh, p1, p2, nb, log, mix=mix)

    @staticmethod
    def backward(ctx, grad_out):
        lin, lout, sh, p1, p2, nb, log, mix = ctx.cfg
        features, radial_table, dist = ctx.saved_tensors
        gf, gt, gd = ops.block_diagonal_bwd(grad_out.contiguous(), features.detach(), radial_table.detach(),
                                            dist.detach(), list(lin), list(lout), sh, p1, p2, nb, log,
                                            mix="bf16" if mix == "bf16" else "bf16x3")
        return (gf if ctx.needs_input_grad[0] else None, gt if ctx.needs_input_grad[1] else None,
                gd if ctx.needs_input_grad[2] else None, None)
