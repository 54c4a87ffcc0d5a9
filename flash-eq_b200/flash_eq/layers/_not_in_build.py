"""Names of the reference package that are outside the edge-message path.

They import (so ``from flash_eq import ...`` keeps working) but raise on use:
the S^2 / Lebedev activation (needs sphericart) and the sequence-distance edge
encoding are not part of this build.
"""
from __future__ import annotations

import torch.nn as nn


def _unavailable(name: str):
    msg = (f"{name} is not part of flash-eq B200 (it is outside the edge-message path: "
           "basis, edgewise linear, attention, pooling, transformer blocks).")

    class _Missing(nn.Module):
        def __init__(self, *args, **kwargs):
            raise NotImplementedError(msg)

    _Missing.__name__ = _Missing.__qualname__ = name

    return _Missing


S2Activation = _unavailable("S2Activation")
SeparableS2Activation = _unavailable("SeparableS2Activation")
SequencePositionEncoding = _unavailable("SequencePositionEncoding")
S2Grid = _unavailable("S2Grid")


def real_spherical_harmonics(*args, **kwargs):
    raise NotImplementedError("real_spherical_harmonics is not part of flash-eq B200 (needs sphericart).")


def lebedev_grid(*args, **kwargs):
    raise NotImplementedError("lebedev_grid is not part of flash-eq B200.")

