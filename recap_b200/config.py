"""Operator settings read by the corrected sparse attention operator.

``OperatorConfig`` has the fields, defaults and validation of the reference's
``recap.config.OperatorConfig`` (recap/config.py:56-80), so a reference ``RecapConfig``'s
``operator`` section can be passed to this package's ``Operator`` unchanged (any object
with these attributes is accepted).
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class OperatorConfig:
    """Sparse attention settings."""

    head_density: float = 0.10  # fraction of key blocks selected per query block
    closure_gate_theta: float = 2.0  # gate of the key-variance correction (nats)
    closure_rank: int = 4  # rank of the per-block key variance
    rerank_min_overlap: float = 0.95
    host_banks: bool = False
    prefetch_banks: bool = True
    bank_chunks: int = 1

    block_size: int = 128

    def validate(self) -> "OperatorConfig":
        if not 0.0 < self.head_density < 1.0:
            raise ValueError("head_density must be in (0,1)")
        if self.closure_gate_theta <= 0:
            raise ValueError("closure_gate_theta must be positive")
        if self.closure_rank < 0:
            raise ValueError("closure_rank must be non-negative")
        if not 0.0 <= self.rerank_min_overlap <= 1.0:
            raise ValueError("rerank_min_overlap must lie in [0,1]")
        if self.bank_chunks < 1:
            raise ValueError("bank_chunks must be at least 1")
        if self.block_size != 128:
            raise ValueError("the exact block-sparse kernel requires block_size=128")
        return self


def keep_blocks(head_density: float, n_blocks: int) -> int:
    """Key blocks kept per query block: ``max(1, round(density * n))`` with Python's
    round-half-to-even (recap/sparse/attention.py:84)."""
    return max(1, round(float(head_density) * n_blocks))
