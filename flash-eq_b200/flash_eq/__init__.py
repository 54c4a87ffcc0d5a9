"""flash-eq on B200: drop-in replacement for the hmblair/flash-eq edge-message path.

Same public names, signatures and parameter layouts as the reference package;
the per-edge work (Wigner-D basis, edgewise linear, attention softmax, pooling)
runs in hand-written sm_100a kernels (libflasheq_b200.so) called through a C ABI.
"""
from .cuda import CUDANotAvailableError
from .graph import Graph
from .layers import (
    EquivariantAttention,
    EquivariantEdgeAttention,
    EquivariantEdgewiseLinear,
    EquivariantGating,
    EquivariantLayerNorm,
    EquivariantLinear,
    EquivariantTransformer,
    EquivariantTransformerBlock,
    GraphPooling,
    RepNorm,
    S2Activation,
    SeparableEquivariantLayerNorm,
    SeparableS2Activation,
    SequencePositionEncoding,
)
from .layers._not_in_build import S2Grid, lebedev_grid, real_spherical_harmonics
from .patch import patch
from .layers.radial import RadialBasisFunctions, RadialMLP, SeparableRadialNet
from .representations import Irrep, ProductIrrep, ProductRepr, Repr, WignerD, WignerDBasis, random_rotation

__version__ = "0.1.0+b200"

__all__ = [
    "Irrep", "ProductIrrep", "Repr", "ProductRepr", "WignerD", "random_rotation", "Graph",
    "EquivariantEdgewiseLinear", "EquivariantAttention", "RepNorm", "EquivariantLinear", "EquivariantGating",
    "EquivariantLayerNorm", "SeparableEquivariantLayerNorm", "GraphPooling", "EquivariantEdgeAttention",
    "S2Activation", "SeparableS2Activation", "EquivariantTransformerBlock", "EquivariantTransformer",
    "WignerDBasis", "RadialBasisFunctions", "RadialMLP", "SeparableRadialNet", "SequencePositionEncoding",
    "S2Grid", "real_spherical_harmonics", "lebedev_grid", "CUDANotAvailableError", "patch",
]
