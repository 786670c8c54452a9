"""Token layout and per-layer sparse state of the operator."""

from .attention import SparseAttention, SparseGeometry
from .geometry import hilbert_permutation, validate_permutation
from .layout import Layout

__all__ = ["Layout", "SparseAttention", "SparseGeometry", "hilbert_permutation", "validate_permutation"]
