"""Quantizer stage: hybrid min-max, fused Hadamard+min-max, centred codebook."""
from .kvserve_quantizer import KVServeQuantizer
from .fused_quantizer import FusedHadamardQuantizer
from .centered_codebook import CenteredCodebookQuantizer

# Config name kept for profile compatibility with the reference.
TileLangFusedQuantizer = FusedHadamardQuantizer

__all__ = ["KVServeQuantizer", "FusedHadamardQuantizer", "CenteredCodebookQuantizer", "TileLangFusedQuantizer"]
