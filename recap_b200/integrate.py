"""Route an installed RECAP (lyraxtg/RECAP, package ``recap``) through this operator.

``use_recap_b200()`` replaces the operator classes the reference's model integrations
build (``recap/models/{cogvideox,wan,hunyuan}.py`` call ``Operator.build`` and, with
``operator.host_banks``, ``recap.host_banks.HostBankOperator``) and lifts their
``block_sparse_attn`` availability check, which this operator does not need.  After it,
``recap.install(pipe, cfg)``, ``session.reset()`` and every ``operator.attend`` call run
unchanged on this package.  The reference's ``Layout`` and ``SparseGeometry`` objects are
used as they are (including the per-prompt text retargeting of the Hunyuan integration).
"""

from __future__ import annotations

import importlib

from .host_banks import HostBankOperator
from .operator import Operator

MODEL_MODULES = ("recap.models.cogvideox", "recap.models.wan", "recap.models.hunyuan")


def _available() -> bool:
    return True


def use_recap_b200() -> list[str]:
    """Patch the installed ``recap`` package; returns the modules patched."""
    import recap
    import recap.host_banks as host_banks
    import recap.operator as operator

    patched = []
    operator.Operator = Operator
    recap.Operator = Operator
    host_banks.HostBankOperator = HostBankOperator
    patched += ["recap.operator", "recap.host_banks"]
    for name in MODEL_MODULES:
        try:
            mod = importlib.import_module(name)
        except ImportError:
            continue
        mod.Operator = Operator
        if hasattr(mod, "block_sparse_available"):
            mod.block_sparse_available = _available
        patched.append(name)
    return patched
