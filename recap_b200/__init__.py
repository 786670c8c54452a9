"""RECAP's corrected sparse attention operator on NVIDIA B200 (sm_100a).

Drop-in for the operator layer of RECAP (``recap.operator.Operator``,
``recap.host_banks.HostBankOperator``, ``recap.sparse``): same classes, signatures and
state machine, with every tensor operation in hand-written sm_100a kernels behind the C
ABI of ``include/recap_b200.h`` (``librecap_b200.so``).  Build the library with
``python -m recap_b200.build``.
"""

from .config import OperatorConfig, keep_blocks
from .host_banks import HostBankOperator
from .operator import EXACT, REFRESH, SPARSE, DetailBank, Operator
from .sparse import Layout, SparseAttention, SparseGeometry, hilbert_permutation

__all__ = [
    "EXACT",
    "REFRESH",
    "SPARSE",
    "DetailBank",
    "HostBankOperator",
    "Layout",
    "Operator",
    "OperatorConfig",
    "SparseAttention",
    "SparseGeometry",
    "hilbert_permutation",
    "keep_blocks",
]
