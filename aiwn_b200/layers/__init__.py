from .indexed_linear import IndexedLinear, indexed_dims, indexed_lr
from .indexed_linear_v2 import GaussianCDFNorm, IndexedLinearV2
from .standard_linear import StandardLinear

__all__ = ["IndexedLinear", "indexed_dims", "indexed_lr", "StandardLinear", "GaussianCDFNorm", "IndexedLinearV2"]
