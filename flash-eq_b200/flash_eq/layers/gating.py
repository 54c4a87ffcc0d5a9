"""Norm-based gating (flash_eq/layers/gating.py:17-76 in the reference).

Without autograd tracking on CUDA float32 inputs the irrep norms and the sigmoid gate are
native kernels (csrc/feq_node.cu); the (C * nreps)^2 linear between them runs on the tensor
cores (csrc/feq_dense.cu) where its size allows.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..representations import Repr
from ..utils import init_linear_weights
from .norm import RepNorm, native_node_ok


class EquivariantGating(nn.Module):
    """x * sigmoid(Linear(irrep norms)) broadcast over each irrep's components."""

    def __init__(self, repr: Repr) -> None:
        super().__init__()
        self.repr = repr
        self.norm = RepNorm(repr)
        n = repr.nreps() * repr.mult
        self.linear = nn.Linear(n, n)
        self.register_buffer("ix", torch.tensor(repr.indices(), dtype=torch.long))
        self.outdims = (repr.mult, repr.nreps())
        self.activation = nn.Sigmoid()
        self.apply(init_linear_weights)

    def forward(self, st: torch.Tensor) -> torch.Tensor:
        norms = self.norm(st)
        *b, _, _ = norms.size()
        if native_node_ok(st, self.linear.weight, self.linear.bias):
            from ..cuda import ops

            # norms and the gate run natively; the dense (C * nreps)^2 linear on the tensor cores
            # (bf16x3) where the kernel serves its size, else a library GEMM
            flat = norms.flatten(-2, -1)
            w = self.linear.weight
            if ops.dense_linear_tc_supported(w.shape[0], w.shape[1]):
                z = ops.dense_linear(flat, w, self.linear.bias)
            else:
                z = self.linear(flat)
            return ops.node_gate(st, z, self.norm._lvals)
        g = self.activation(self.linear(norms.flatten(-2, -1)).view(*b, *self.outdims))
        return st * g[..., self.ix]
