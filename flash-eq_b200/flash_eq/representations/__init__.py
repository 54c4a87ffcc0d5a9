"""SO(3) representations and Wigner-D bases (same names as the reference package)."""
from .types import Irrep, ProductIrrep, ProductRepr, Repr
from .wigner import LazyBasis, WignerD, WignerDBasis, random_rotation

__all__ = ["Irrep", "ProductIrrep", "Repr", "ProductRepr", "WignerD", "WignerDBasis", "random_rotation",
           "LazyBasis"]
