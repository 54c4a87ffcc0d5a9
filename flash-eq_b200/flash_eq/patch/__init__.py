"""flash_eq.patch: NVIDIA SE(3)-Transformer layers on the flash-eq edge kernel
(flash_eq/patch/__init__.py in the reference).

``PatchedConvSE3`` (the replacement convolution, reference _patched_conv.py:21-129) is part of
this build and runs on the B200 kernels: given a converted radial table it takes the same
inputs as the reference's.  ``patch(model)`` -- finding ConvSE3 modules in an NVIDIA model
and converting their radial networks into tables (reference __init__.py:104-229,
_conversion.py, _convention.py) -- needs NVIDIA's SE(3)-Transformer, DGL and the
Lebedev-quadrature Clebsch-Gordan projection (sphericart convention), none of which is part
of this build; it raises with that explanation.
"""
from __future__ import annotations

from ._patched_conv import PatchedConvSE3

__all__ = ["patch", "PatchedConvSE3"]


def patch(model, num_bins: int = 500, min_dist: float = 0.0, max_dist: float = 10.0, dtype=None):
    """Convert every NVIDIA ``ConvSE3`` of ``model`` (reference flash_eq/patch/__init__.py:104-229).

    Not available in this build: the weight conversion projects NVIDIA's Clebsch-Gordan radial
    kernels onto the Wigner-D block layout with a Lebedev-quadrature real-SH basis
    (sphericart convention), which this build does not include.  Construct
    ``PatchedConvSE3`` from an already converted table instead."""
    raise NotImplementedError(
        "flash_eq.patch.patch: converting NVIDIA ConvSE3 weights (Clebsch-Gordan projection on a Lebedev "
        "grid, sphericart convention) is not part of flash-eq B200; build PatchedConvSE3 from a converted "
        "(num_bins + 1, C_out, C_in, W) table instead")
