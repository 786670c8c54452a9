"""End-to-end parity of recap_b200.Operator (REFRESH -> SPARSE -> revalidating REFRESH)
against the CPU oracle on the same bf16-rounded inputs, and against the golden outputs
the reference produced in fp32 (tests/golden/make_golden.py).

Tolerances (from the benchmark's parity criteria): bf16 outputs within max-abs 2e-2 and
mean-rel 1e-2, the max-abs bound scaled by the output magnitude where that exceeds 1 (one
bf16 ulp is 2^-5 = 0.031 for values in [4, 8)); selected blocks bit-exact except
documented fp ties (see test_gpu_kernels._selection_matches); e_detail within 2e-2
relative."""

import math

import pytest
import torch

from oracle import recap_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"
MAX_ABS = 2e-2
MEAN_REL = 1e-2


def _build(spec, **kw):
    from recap_b200 import Operator, OperatorConfig
    from recap_b200.sparse import Layout, SparseGeometry, hilbert_permutation

    perm = hilbert_permutation(spec["grid"])
    layout = Layout.from_permutation(perm, text_tokens=spec["text"], text_first=spec["text_first"])
    geo = SparseGeometry.build(layout, 128)
    cfg = OperatorConfig(head_density=spec["density"], **kw)
    return Operator.build(cfg, geo, n_layers=1), perm


def _mean_rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a - b).abs().mean() / b.abs().mean().clamp_min(1e-30))


def _inputs(spec):
    if spec["inputs"] == "iid":
        return orc.config1_inputs(0)
    return orc.smooth_lowrank(spec["grid"], spec["heads"], spec["dim"], spec["text"], spec["text_first"], seed=0,
                              dtype=torch.float32)


SPECS = {
    "config1": dict(grid=(8, 16, 16), text=0, text_first=False, heads=2, dim=64, density=0.25, inputs="iid"),
    "textfirst_partial": dict(grid=(3, 12, 20), text=50, text_first=True, heads=2, dim=64, density=0.34,
                              inputs="smooth"),
    "textlast_d128": dict(grid=(4, 9, 14), text=40, text_first=False, heads=2, dim=128, density=0.5,
                          inputs="smooth"),
    "video_d128": dict(grid=(2, 16, 32), text=0, text_first=False, heads=2, dim=128, density=0.25,
                       inputs="smooth"),
}


def _run_both(spec):
    """Run the GPU operator and the bf16 oracle through refresh/sparse/refresh."""
    from recap_b200 import REFRESH, SPARSE

    op, perm = _build(spec)
    bf = torch.bfloat16
    q0, k0, v0 = (t.to(bf) for t in _inputs(spec))
    q1, k1, v1 = orc.perturb3(q0.float(), k0.float(), v0.float(), seed=1)
    q2, k2, v2 = orc.perturb3(q1, k1, v1, seed=2)
    q1, k1, v1, q2, k2, v2 = (t.to(bf) for t in (q1, k1, v1, q2, k2, v2))
    res = {}
    op.begin_step(0, REFRESH)
    res["r0"] = op.attend(0, *(t.to(DEV) for t in (q0, k0, v0))).cpu()
    bank = op.banks[0][0]
    res["r0_partition"] = bank.partition.cpu().clone()
    res["r0_value"] = bank.value.cpu().clone()
    res["r0_log_mass"] = bank.log_mass.cpu().clone()
    res["r0_coarse_lse"] = bank.coarse_lse.cpu().clone()
    basis = op.layers[0][0].basis.cpu().clone()
    op.begin_step(1, SPARSE)
    res["s1"] = op.attend(0, *(t.to(DEV) for t in (q1, k1, v1))).cpu()
    op.begin_step(2, REFRESH)
    res["r2"] = op.attend(0, *(t.to(DEV) for t in (q2, k2, v2))).cpu()
    res["r2_validation"] = op.drain_validation()
    res["r2_partition"] = bank.partition.cpu().clone()
    op.check_device_status()

    oracle = orc.OracleOperator(perm, spec["text"], spec["text_first"], head_density=spec["density"], dtype=bf,
                                basis_override=basis)
    ref = {}
    ref["r0"] = oracle.refresh(0, q0[0].float(), k0[0].float(), v0[0].float())
    st = oracle.layer(0)
    ref["r0_partition"] = st.partition.clone()
    ref["r0_value"] = st.value.clone()
    ref["r0_log_mass"] = st.log_mass.clone()
    ref["r0_coarse_lse"] = st.coarse_lse.clone()
    oracle.step = 1
    ref["s1"] = oracle.sparse(0, q1[0].float(), k1[0].float(), v1[0].float())
    oracle.step = 2
    ref["r2"] = oracle.refresh(0, q2[0].float(), k2[0].float(), v2[0].float())
    ref["r2_validation"] = oracle.drain_validation()
    ref["r2_partition"] = st.partition.clone()
    return res, ref, op


@pytest.mark.parametrize("name", list(SPECS))
def test_operator_matches_oracle(name):
    spec = SPECS[name]
    res, ref, _ = _run_both(spec)
    heads = spec["heads"]
    assert torch.equal(res["r0_partition"].reshape(heads, *res["r0_partition"].shape[-2:]), ref["r0_partition"])
    for key in ("r0", "s1", "r2"):
        got = res[key][0].float()
        exp = ref[key].float()
        err = float((got - exp).abs().max())
        bound = MAX_ABS * max(1.0, float(exp.abs().max()))
        assert err <= bound, f"{key}: max abs {err} > {bound}"
        assert _mean_rel(got, exp) <= MEAN_REL, f"{key}: mean rel {_mean_rel(got, exp)}"
    assert (res["r0_log_mass"] - ref["r0_log_mass"]).abs().max() <= 5e-2
    assert (res["r0_coarse_lse"] - ref["r0_coarse_lse"]).abs().max() <= 5e-3
    det_err = (res["r0_value"].float() - ref["r0_value"].float()).abs()
    assert _mean_rel(res["r0_value"].float(), ref["r0_value"].float()) <= 5e-2, float(det_err.max())
    age, err = res["r2_validation"]
    rage, rerr = ref["r2_validation"]
    assert age == rage
    assert abs(err - rerr) <= 2e-2 * rerr, (err, rerr)
    assert torch.equal(res["r2_partition"].reshape(heads, *res["r2_partition"].shape[-2:]), ref["r2_partition"])


@pytest.mark.parametrize("name", list(SPECS))
def test_operator_matches_reference_golden(golden_dir, name):
    """GPU bf16 run against the reference's own fp32 outputs (looser: the inputs differ by
    bf16 rounding)."""
    from recap_b200 import REFRESH, SPARSE

    g = torch.load(golden_dir / f"{name}.pt")
    spec = g["spec"]
    op, _ = _build(spec)
    q0, k0, v0 = _inputs(spec)
    q1, k1, v1 = orc.perturb3(q0, k0, v0, seed=1)
    op.begin_step(0, REFRESH)
    op.attend(0, *(t.to(DEV) for t in (q0, k0, v0)))  # fp32 in: cast to bf16 inside
    part = op.banks[0][0].partition.cpu()[0]
    gpart = g["r0_partition"][0]
    overlap = float((part & gpart).sum()) / float(gpart.sum())
    assert overlap >= 0.9, overlap  # bf16 inputs can move near-tied blocks
    op.begin_step(1, SPARSE)
    out = op.attend(0, *(t.to(DEV) for t in (q1, k1, v1))).cpu()[0]
    assert out.dtype == torch.float32
    ref = g["s1_out"][0]
    assert _mean_rel(out, ref) <= 2e-2, _mean_rel(out, ref)
    # rows whose query block selected the same key blocks as the reference must agree
    # closely; other rows use a different (equally valid) sparse approximation
    perm = torch.as_tensor(op.layout.permutation)
    fwd, inv = orc.gather_indices(perm, spec["text"], spec["text_first"])
    nb = part.shape[-1]
    same_block = (part == gpart).all(-1)  # [heads, nB]
    qblock = inv // 128  # native row -> reordered query block
    rows_ok = torch.zeros(spec["heads"], out.shape[1], dtype=torch.bool)
    for h in range(spec["heads"]):
        video_q = qblock < nb
        ok = torch.ones_like(qblock, dtype=torch.bool)
        ok[video_q] = same_block[h][qblock[video_q]]
        rows_ok[h] = ok
    assert rows_ok.float().mean() >= 0.5
    # bf16-rounded inputs move softmax rows with large logits (these smooth inputs give
    # |q.k| s ~ 10), so against the fp32 reference only the mean error is bounded here;
    # the elementwise bound is checked against the oracle on the same bf16 inputs above.
    assert _mean_rel(out[rows_ok], ref[rows_ok]) <= 2e-2


def test_sparse_before_refresh_raises():
    from recap_b200 import SPARSE

    op, _ = _build(SPECS["config1"])
    op.begin_step(0, SPARSE)
    q = torch.zeros(1, 2, 2048, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError):
        op.attend(0, q, q, q)


def test_exact_matches_dense_attention():
    from recap_b200 import EXACT

    op, _ = _build(SPECS["textfirst_partial"])
    op.begin_step(0, EXACT)
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 770, 64, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3))
    out = op.attend(0, q, k, v).float()
    ref = torch.softmax((q.float() @ k.float().transpose(-1, -2)) / 8.0, -1) @ v.float()
    assert float((out - ref).abs().max()) <= MAX_ABS


@pytest.mark.parametrize("prefetch,slots", [(True, 2), (False, 1), (True, 3)])
def test_host_bank_streaming_matches_resident(prefetch, slots):
    """HostBankOperator with an HBM budget of zero streams each layer's refinement through
    pinned host memory (a ring of device slots, prefetch and write-back streams); its
    outputs equal the HBM-resident operator's bit for bit over refresh -> sparse -> sparse
    -> refresh across three layers (the copies are exact and the kernels are the same)."""
    from recap_b200 import REFRESH, SPARSE, HostBankOperator, Operator, OperatorConfig
    from recap_b200.sparse import Layout, SparseGeometry, hilbert_permutation

    spec = SPECS["textlast_d128"]
    perm = hilbert_permutation(spec["grid"])
    layout = Layout.from_permutation(perm, text_tokens=spec["text"], text_first=spec["text_first"])
    geo = SparseGeometry.build(layout, 128)
    cfg = OperatorConfig(head_density=spec["density"])
    n_layers = 3
    resident = Operator.build(cfg, geo, n_layers=n_layers)
    streamed = HostBankOperator.build(cfg, geo, n_layers=n_layers)
    streamed.hbm_budget = 0
    streamed.ring_slots = slots
    streamed.set_prefetch(prefetch)
    held = streamed.preallocate_host(n_layers, spec["heads"], spec["dim"])
    assert streamed.resident is False and held > 0

    bf = torch.bfloat16
    base = [t.to(bf) for t in _inputs(spec)]
    steps = [REFRESH, SPARSE, SPARSE, REFRESH]
    for step, kind in enumerate(steps):
        for op in (resident, streamed):
            op.begin_step(step, kind)
        for layer in range(n_layers):
            q, k, v = orc.perturb3(*(t.float() for t in base), seed=100 * step + layer)
            args = [t.to(bf).to(DEV) for t in (q, k, v)]
            out_r = resident.attend(layer, *args)
            out_s = streamed.attend(layer, *args)
            assert torch.equal(out_r, out_s), (step, layer)
    streamed.finish()
    resident.check_device_status()
    streamed.check_device_status()
