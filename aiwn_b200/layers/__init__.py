from .indexed_linear import IndexedLinear, indexed_dims, indexed_lr
from .standard_linear import StandardLinear

__all__ = ["IndexedLinear", "indexed_dims", "indexed_lr", "StandardLinear"]
