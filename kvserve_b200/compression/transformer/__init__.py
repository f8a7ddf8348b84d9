"""Transform stage: random-sign Hadamard, signed DCT-II, Haar rotation."""
from .hadamard import HadamardTransform
from .orthogonal import OrthogonalTransform
from .kvserve_transformer import KVServeTransformer

__all__ = ["HadamardTransform", "OrthogonalTransform", "KVServeTransformer"]
