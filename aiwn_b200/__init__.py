"""aiwn_b200 -- B200-native (sm_100a) IndexedLinear, a drop-in for the
reference package's ``aiwn.layers.indexed_linear`` hot path."""
from .layers import GaussianCDFNorm, IndexedLinear, IndexedLinearV2, StandardLinear, indexed_dims, indexed_lr
from .layers.indexed_linear import TRITON_OK, _Fn, triton_available

__all__ = ["IndexedLinear", "IndexedLinearV2", "GaussianCDFNorm", "StandardLinear", "indexed_dims", "indexed_lr",
           "TRITON_OK", "triton_available", "_Fn"]
