"""Wiring of recap_b200 into the reference package.  Runs where the environment variable
RECAP_REFERENCE_PATH names a checkout of the reference tree (lyraxtg/RECAP), and is
skipped elsewhere.  No GPU: only construction and the host-side state machine are
exercised."""

import os
import sys
from pathlib import Path

import pytest

_REF_ENV = os.environ.get("RECAP_REFERENCE_PATH")
REF = Path(_REF_ENV) if _REF_ENV else None
pytestmark = pytest.mark.skipif(REF is None or not (REF / "recap" / "__init__.py").exists(),
                                reason="RECAP_REFERENCE_PATH does not name a reference checkout")


@pytest.fixture(scope="module")
def recap_pkg():
    sys.path.insert(0, str(REF))
    import recap

    from recap_b200.integrate import use_recap_b200

    patched = use_recap_b200()
    yield recap, patched


def test_models_build_our_operator(recap_pkg):
    recap, patched = recap_pkg
    import recap.models.wan as wan

    import recap_b200

    assert "recap.models.wan" in patched
    assert wan.Operator is recap_b200.Operator
    assert wan.block_sparse_available()
    import recap.host_banks as hb

    assert hb.HostBankOperator is recap_b200.HostBankOperator


def test_session_drives_our_operator_state_machine(recap_pkg):
    recap, _ = recap_pkg
    from recap.config import load_config
    from recap.session import RecapSession
    from recap.sparse.attention import SparseGeometry as RefGeometry
    from recap.sparse.geometry import hilbert_permutation
    from recap.sparse.layout import Layout as RefLayout

    import recap_b200

    cfg = load_config(REF / "configs" / "hunyuan_fast.json")
    layout = RefLayout.from_permutation(hilbert_permutation((2, 8, 8)), text_tokens=16, text_first=False)
    geo = RefGeometry.build(layout, 128)
    op = recap_b200.Operator.build(cfg.operator, geo, n_layers=3, n_streams=1)
    session = RecapSession(cfg, op, calls_per_step=1)
    assert op.kind == recap_b200.EXACT and not op.banks_valid
    action = session.begin(0)
    assert action in (recap_b200.EXACT, recap_b200.REFRESH)
    assert op.drain_validation() is None
    session.reset()
    assert op.step == 0 and op.stream == 0


def test_reference_layout_indices_and_retarget(recap_pkg):
    import torch
    from recap.models.hunyuan import retarget_text_tokens
    from recap.sparse.geometry import hilbert_permutation
    from recap.sparse.layout import Layout as RefLayout

    from recap_b200.sparse.layout import gather_rows

    layout = RefLayout.from_permutation(hilbert_permutation((2, 8, 8)), text_tokens=16, text_first=False)
    cpu = torch.device("cpu")
    rows = gather_rows(layout, cpu)
    x = torch.randn(1, 1, 144, 4)
    assert torch.equal(x[..., rows.long(), :], layout.reorder(x))
    retarget_text_tokens(layout, 9)
    rows = gather_rows(layout, cpu)
    assert rows.numel() == 137
    y = torch.randn(1, 1, 137, 4)
    assert torch.equal(y[..., rows.long(), :], layout.reorder(y))
