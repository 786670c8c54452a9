"""3-D Hilbert order of the video tokens (host side, computed once per model).

Each 128-token block of the reordered sequence is then a compact spatio-temporal region.
The order must be integer-identical to the reference's ``hilbert_permutation``
(recap/sparse/geometry.py:27-67): x is the leading axis, y the second, t the third; the
Hilbert index is John Skilling's transposed form ("Programming the Hilbert curve",
AIP Conf. Proc. 707, 2004) interleaved most significant bit first, and tokens are ordered
by a stable sort of that index.
"""

from __future__ import annotations

import math
from typing import Sequence

import numpy as np


def validate_permutation(permutation: np.ndarray, grid: Sequence[int]) -> np.ndarray:
    """Check a reordered-position -> native-index permutation of ``prod(grid)`` tokens."""
    n = int(np.prod([int(g) for g in grid]))
    perm = np.asarray(permutation, dtype=np.int64)
    if perm.shape != (n,):
        raise ValueError(f"permutation shape {perm.shape} != ({n},)")
    if perm.min(initial=0) != 0 or perm.max(initial=-1) != n - 1:
        raise ValueError("permutation is outside [0, prod(grid))")
    if np.unique(perm).size != n:
        raise ValueError("permutation is not one-to-one")
    return perm


def _transposed_hilbert(coords: np.ndarray, order: int) -> np.ndarray:
    """Skilling's axes-to-transpose on a [dims, n] int64 array (modified in place)."""
    dims = coords.shape[0]
    bit = 1 << (order - 1)
    # inverse "undo excess work", most significant bit down to bit 1
    while bit > 1:
        lower = bit - 1
        for axis in range(dims):
            on = (coords[axis] & bit) != 0
            coords[0] = np.where(on, coords[0] ^ lower, coords[0])
            exchange = np.where(on, 0, (coords[0] ^ coords[axis]) & lower)
            coords[0] ^= exchange
            coords[axis] ^= exchange
        bit >>= 1
    # Gray encode
    for axis in range(1, dims):
        coords[axis] ^= coords[axis - 1]
    fold = np.zeros_like(coords[0])
    bit = 1 << (order - 1)
    while bit > 1:
        fold = np.where((coords[dims - 1] & bit) != 0, fold ^ (bit - 1), fold)
        bit >>= 1
    coords ^= fold[None, :]
    return coords


def hilbert_permutation(grid: Sequence[int]) -> np.ndarray:
    """Reordered position -> native token index (``t*H*W + y*W + x``) along a 3-D Hilbert
    curve over ``grid = (T, H, W)``."""
    frames, height, width = (int(g) for g in grid)
    order = max(1, math.ceil(math.log2(max(frames, height, width))))
    t, y, x = np.meshgrid(np.arange(frames), np.arange(height), np.arange(width), indexing="ij")
    native = (t * (height * width) + y * width + x).reshape(-1)
    coords = np.stack([x.reshape(-1), y.reshape(-1), t.reshape(-1)]).astype(np.int64)
    coords = _transposed_hilbert(coords, order)
    key = np.zeros(coords.shape[1], dtype=np.int64)
    for b in range(order - 1, -1, -1):
        for axis in range(3):
            key = (key << 1) | ((coords[axis] >> b) & 1)
    return validate_permutation(native[np.argsort(key, kind="stable")], grid)
