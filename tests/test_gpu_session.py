"""The reference's own step loop driving this operator on the GPU: ``recap.session.RecapSession``
(the per-step EXACT / REFRESH / SPARSE / REUSE decisions, the prediction cache, the validation
of each refreshed correction) wraps a small two-layer transformer whose attention calls go to
``recap_b200.Operator.attend``, as the reference's model integrations route them after
``recap_b200.integrate.use_recap_b200()``.

The reference package is imported from ``baseline/_ref`` (an offline ``pip install --no-deps
--target baseline/_ref`` of lyraxtg/RECAP, git-ignored); the test is skipped where that
install or a GPU is missing.  EXACT and REFRESH calls are checked against fp32 dense
attention on the same Q/K/V (max-abs 2e-2, the bf16 tolerance of the other tests).  The
REFRESH and SPARSE calls of every layer, in the order the session made them, are replayed
through the CPU oracle (``oracle.recap_oracle.OracleOperator``, each layer seeded with this
operator's closure basis): every output within max-abs 2e-2 (scaled by the output magnitude
above 1) and mean-rel 1e-2, and every validation error the session received within 2e-2
relative of the oracle's, with the same correction age.  The trajectory moves far between
refreshes on purpose, so the session fails some validations and re-decides; the SPARSE
estimates are then far from dense attention, which is why they are checked against the
oracle and not against dense attention."""

import json
import math
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
H, D, GRID, TEXT, LAYERS, STEPS = 2, 128, (4, 8, 16), 64, 2, 20


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.skipif(not (REF / "recap" / "session.py").exists(), reason="no reference install in baseline/_ref")
def test_reference_session_drives_operator():
    sys.path.insert(0, str(REF))
    from recap.config import PACKAGE_DIR, _from_profile
    from recap.session import RecapSession
    from recap.sparse.attention import SparseGeometry as RefGeometry
    from recap.sparse.geometry import hilbert_permutation
    from recap.sparse.layout import Layout as RefLayout

    import recap_b200
    from recap_b200.integrate import use_recap_b200

    use_recap_b200()
    dev = torch.device("cuda", 0)
    # the HunyuanVideo fast profile on a small grid, HBM banks, 20 steps
    prof = json.loads((PACKAGE_DIR / "profiles" / "hunyuan_fast.json").read_text())
    prof["geometry"].update(grid=list(GRID), text_tokens=TEXT)
    prof["operator"].update(host_banks=False, prefetch_banks=False)
    prof["schedule"].update(num_steps=STEPS)
    cfg = _from_profile("hunyuan", prof)
    layout = RefLayout.from_permutation(hilbert_permutation(GRID), text_tokens=TEXT, text_first=False)
    geo = RefGeometry.build(layout, 128)
    op = recap_b200.Operator.build(cfg.operator, geo, n_layers=LAYERS, n_streams=1)
    S = layout.video_tokens + TEXT

    g = torch.Generator().manual_seed(0)
    weights = [(torch.randn(H * D, 3 * H * D, generator=g) / (H * D) ** 0.5).to(dev) for _ in range(LAYERS)]
    checks = []
    calls = []  # (step, kind, layer, q, k, v, output) of every computed attention call

    class TwoLayers(torch.nn.Module):
        def forward(self, x, timestep=None):
            for i, w in enumerate(weights):
                qkv = (x @ w).view(1, S, 3, H, D).permute(2, 0, 3, 1, 4).to(torch.bfloat16)
                q, k, v = qkv[0], qkv[1], qkv[2]
                o = op.attend(i, q, k, v)
                ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
                err = (o.float() - ref)
                checks.append((op.kind, float(err.abs().max()),
                               float(err.norm() / ref.norm().clamp_min(1e-30)), bool(torch.isfinite(o).all())))
                calls.append((op.step, op.kind, i, q[0].cpu(), k[0].cpu(), v[0].cpu(), o[0].cpu()))
                x = x + o.float().permute(0, 2, 1, 3).reshape(1, S, H * D)
            return x

    model = TwoLayers()
    session = RecapSession(cfg, op, calls_per_step=1)
    session.install(model)
    x0 = torch.randn(1, S, H * D, generator=g)
    dirs = [torch.randn(1, S, H * D, generator=g) for _ in range(3)]
    for t in range(STEPS):
        s = t / STEPS
        x = x0 + 0.3 * (s * dirs[0] + s * s * dirs[1] + 2.0 * torch.sin(torch.tensor(20.0 * s)) * dirs[2])
        model(x.to(dev))
    op.check_device_status()
    torch.cuda.synchronize()

    actions = [row["a"] for row in session.actions]
    print("actions:", actions)
    print("validations:", session.controller.validations)
    by_kind = {}
    for kind, max_abs, rel, finite in checks:
        by_kind.setdefault(kind, []).append((max_abs, rel))
        assert finite, f"non-finite {kind} output"
    for kind, rows in by_kind.items():
        print(kind, "calls", len(rows), "max-abs", max(r[0] for r in rows), "rel-rms", max(r[1] for r in rows))
    assert {"exact", "refresh", "sparse", "reuse"} <= set(actions), actions
    for kind in ("exact", "refresh"):
        worst = max(r[0] for r in by_kind[kind])
        assert worst <= 2e-2, f"{kind} output differs from dense attention by {worst}"
    assert session.controller.validations, "no refreshed correction was validated"

    # the same REFRESH / SPARSE history through the CPU oracle
    from oracle import recap_oracle as orc

    oracle = orc.OracleOperator(layout.permutation, TEXT, False, head_density=cfg.operator.head_density,
                                closure_gate_theta=cfg.operator.closure_gate_theta,
                                closure_rank=cfg.operator.closure_rank,
                                rerank_min_overlap=cfg.operator.rerank_min_overlap, dtype=torch.bfloat16)
    for i in range(LAYERS):
        oracle.layer(i).basis = op.layers[0][i].basis.cpu().clone()
    validations = {v["t"]: v for v in session.controller.validations}
    worst = {"refresh": 0.0, "sparse": 0.0}
    checked = []

    def check_validation(step):
        expected = validations.get(step)
        measured = oracle.drain_validation()
        if expected is not None:
            assert measured is not None and measured[0] == expected["age"], (measured, expected)
            assert abs(measured[1] - expected["error"]) <= 2e-2 * measured[1] + 1e-6, (measured, expected)
            checked.append(step)

    last_refresh_step = None
    for step, kind, i, q, k, v, got in calls:
        if kind not in ("refresh", "sparse"):
            continue
        if last_refresh_step is not None and step != last_refresh_step:
            check_validation(last_refresh_step)
            last_refresh_step = None
        oracle.step = step
        exp = (oracle.refresh if kind == "refresh" else oracle.sparse)(i, q.float(), k.float(), v.float()).float()
        if kind == "refresh":
            last_refresh_step = step
        err = float((got.float() - exp).abs().max())
        mean_rel = float((got.float() - exp).abs().mean() / exp.abs().mean().clamp_min(1e-30))
        bound = 2e-2 * max(1.0, float(exp.abs().max()))
        assert err <= bound and mean_rel <= 1e-2, f"step {step} {kind} layer {i}: max-abs {err}, mean-rel {mean_rel}"
        worst[kind] = max(worst[kind], err)
    if last_refresh_step is not None:
        check_validation(last_refresh_step)
    print("against the oracle, worst max-abs:", worst, "validations checked at steps", checked)
    assert sorted(checked) == sorted(validations), (checked, list(validations))
    assert math.isfinite(worst["sparse"])
    session.reset()
    assert op.step == 0 and not op.banks_valid
