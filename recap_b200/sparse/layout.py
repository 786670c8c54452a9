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

    def _indices_cpu(self) -> tuple[torch.Tensor, torch.Tensor]:
        nv, tt = self.video_tokens, self.text_tokens
        text = torch.arange(tt, dtype=torch.long)
        if self.text_first:
            fwd = torch.cat((self.permutation + tt, text))      # [text | video] -> [video_r | text]
            inv = torch.cat((text + nv, self.inverse))
        else:
            fwd = torch.cat((self.permutation, text + nv))      # [video | text] -> [video_r | text]
            inv = torch.cat((self.inverse, text + nv))
        return fwd, inv

    def _gather_indices(self, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        """int64 gather indices (reorder, restore), cached per device."""
        key = f"i64:{device}"
        cached = self._gather_cache.get(key)
        if cached is None:
            fwd, inv = self._indices_cpu()
            cached = (fwd.to(device), inv.to(device))
            self._gather_cache[key] = cached
        return cached

    def gather_rows(self, device: torch.device) -> torch.Tensor:
        """int32 [S]: native token of reordered row r.  Also the native output row of
        reordered row r, since restore is the inverse gather."""
        key = f"rows:{device}"
        cached = self._gather_cache.get(key)
        if cached is None:
            cached = self._indices_cpu()[0].to(torch.int32).to(device)
            self._gather_cache[key] = cached
        return cached

    def video_permutation(self, device: torch.device, dtype: torch.dtype = torch.long) -> torch.Tensor:
        """The video permutation on ``device``, cached."""
        key = f"video:{device}:{dtype}"
        cached = self._gather_cache.get(key)
        if cached is None:
            cached = self.permutation.to(dtype).to(device)
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
