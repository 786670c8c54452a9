"""Native token order <-> [Hilbert-ordered video | text] (recap/sparse/layout.py:14-92).

Same fields and semantics as the reference's ``Layout``.  The operator does not gather
through torch: its layout kernel reads the native tensors through ``gather_rows`` (int32,
cached per device) and its epilogue writes back through the same index, so ``reorder`` and
``restore`` here are conveniences for callers and tests.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch


def _indices_of(layout) -> tuple[torch.Tensor, torch.Tensor]:
    """(reorder, restore) int64 CPU indices from a layout's fields (recap/sparse/layout.py:48-68)."""
    p = torch.as_tensor(layout.permutation, dtype=torch.long, device="cpu")
    inverse = getattr(layout, "inverse", None)
    inverse = torch.argsort(p) if inverse is None else torch.as_tensor(inverse, dtype=torch.long, device="cpu")
    nv, tt = p.numel(), int(layout.text_tokens)
    text = torch.arange(tt, dtype=torch.long)
    if layout.text_first:
        return torch.cat((p + tt, text)), torch.cat((text + nv, inverse))
    return torch.cat((p, text + nv)), torch.cat((inverse, text + nv))


def gather_rows(layout, device: torch.device) -> torch.Tensor:
    """int32 [S]: native token of reordered row r, which is also the native output row of
    reordered row r (restore is the inverse gather).  Works on this package's ``Layout``
    and on the reference's (any object with ``permutation``, ``text_tokens``,
    ``text_first`` and a ``_gather_cache`` dict); cached in ``_gather_cache``, which the
    reference clears when it retargets the text length (recap/models/hunyuan.py:30-39)."""
    cache = layout._gather_cache
    key = f"recap_b200:rows:{device}:{int(layout.text_tokens)}"
    cached = cache.get(key)
    if cached is None:
        cached = _indices_of(layout)[0].to(torch.int32).to(device)
        cache[key] = cached
    return cached


def video_permutation_i32(layout, device: torch.device) -> torch.Tensor:
    """int32 [Nv] reordered video position -> native video index, cached per device."""
    cache = layout._gather_cache
    key = f"recap_b200:video:{device}"
    cached = cache.get(key)
    if cached is None:
        cached = torch.as_tensor(layout.permutation).to(torch.int32).to(device)
        cache[key] = cached
    return cached


def sequence_tokens(layout) -> int:
    return int(layout.video_tokens) + int(layout.text_tokens)


def video_offset(layout) -> int:
    return int(layout.text_tokens) if layout.text_first else 0


@dataclass
class Layout:
    permutation: torch.Tensor  # reordered video position -> native video position (int64, CPU)
    inverse: torch.Tensor
    video_tokens: int
    text_tokens: int
    text_first: bool
    _gather_cache: dict = field(default_factory=dict, repr=False, compare=False)

    @classmethod
    def from_permutation(
        cls,
        permutation: np.ndarray | torch.Tensor,
        *,
        text_tokens: int,
        text_first: bool,
    ) -> "Layout":
        p = torch.as_tensor(permutation, dtype=torch.long, device="cpu")
        if p.ndim != 1 or torch.unique(p).numel() != p.numel():
            raise ValueError("invalid layout permutation")
        return cls(
            permutation=p,
            inverse=torch.argsort(p),
            video_tokens=p.numel(),
            text_tokens=int(text_tokens),
            text_first=bool(text_first),
        )

    @property
    def video_offset(self) -> int:
        """Position of the first video token in the native sequence."""
        return self.text_tokens if self.text_first else 0

    @property
    def sequence_tokens(self) -> int:
        return self.video_tokens + self.text_tokens

    def _gather_indices(self, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        """int64 gather indices (reorder, restore), cached per device."""
        key = f"i64:{device}:{self.text_tokens}"
        cached = self._gather_cache.get(key)
        if cached is None:
            fwd, inv = _indices_of(self)
            cached = (fwd.to(device), inv.to(device))
            self._gather_cache[key] = cached
        return cached

    def gather_rows(self, device: torch.device) -> torch.Tensor:
        return gather_rows(self, device)

    def video_permutation(self, device: torch.device) -> torch.Tensor:
        """The video permutation on ``device`` (int64), cached."""
        key = f"video64:{device}"
        cached = self._gather_cache.get(key)
        if cached is None:
            cached = self.permutation.to(device)
            self._gather_cache[key] = cached
        return cached

    def _check(self, x: torch.Tensor) -> None:
        if x.shape[-2] != self.video_tokens + self.text_tokens:
            raise ValueError(
                f"sequence {x.shape[-2]} != video+text {self.video_tokens + self.text_tokens}"
            )

    def reorder(self, x: torch.Tensor) -> torch.Tensor:
        """Native model order -> [reordered video | text]."""
        self._check(x)
        return x.index_select(-2, self._gather_indices(x.device)[0])

    def restore(self, x: torch.Tensor) -> torch.Tensor:
        """[reordered video | text] -> native model order."""
        self._check(x)
        return x.index_select(-2, self._gather_indices(x.device)[1])
