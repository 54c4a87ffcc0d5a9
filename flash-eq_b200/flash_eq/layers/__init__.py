"""Equivariant layers (same names as the reference's flash_eq.layers)."""
from ._not_in_build import S2Activation, SeparableS2Activation, SequencePositionEncoding
from .attention import EquivariantAttention, EquivariantEdgeAttention
from .gating import EquivariantGating
from .linear import EquivariantEdgewiseLinear, EquivariantLinear
from .norm import EquivariantLayerNorm, RepNorm, SeparableEquivariantLayerNorm
from .pooling import GraphPooling
from .radial import RadialBasisFunctions, RadialMLP, SeparableRadialNet
from .transformer import DropPath, EquivariantTransformer, EquivariantTransformerBlock, LayerScale

__all__ = [
    "EquivariantEdgewiseLinear", "EquivariantLinear", "EquivariantEdgeAttention", "EquivariantAttention",
    "RepNorm", "EquivariantLayerNorm", "SeparableEquivariantLayerNorm", "GraphPooling", "EquivariantGating",
    "S2Activation", "SeparableS2Activation", "EquivariantTransformerBlock", "EquivariantTransformer",
    "RadialBasisFunctions", "RadialMLP", "SeparableRadialNet", "SequencePositionEncoding",
    "LayerScale", "DropPath",
]
