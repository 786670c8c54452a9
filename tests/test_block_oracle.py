"""The block-sampled oracle (oracle/block_oracle.py) against the full oracle
(oracle/recap_oracle.py, pinned to the reference's golden vectors) on CPU: with every
query block chosen it reproduces the full oracle's REFRESH -> SPARSE -> revalidating
REFRESH, outputs, banks and validation error; with a subset it gives the same rows."""

import math

import pytest
import torch

from oracle import block_oracle as bo
from oracle import recap_oracle as orc

SPECS = {
    "textfirst_partial": dict(grid=(3, 12, 20), text=50, text_first=True, heads=2, dim=64, density=0.34),
    "textlast_d128": dict(grid=(4, 9, 14), text=40, text_first=False, heads=2, dim=128, density=0.5),
}


def _inputs(spec):
    bf = torch.bfloat16
    q0, k0, v0 = (t[0].float() for t in orc.smooth_lowrank(spec["grid"], spec["heads"], spec["dim"], spec["text"],
                                                          spec["text_first"], seed=0, dtype=bf))
    q1, k1, v1 = (t.to(bf).float() for t in orc.perturb3(q0, k0, v0, seed=1))
    q2, k2, v2 = (t.to(bf).float() for t in orc.perturb3(q1, k1, v1, seed=2))
    return (q0, k0, v0), (q1, k1, v1), (q2, k2, v2)


def _perm(spec):
    from recap_b200.sparse import hilbert_permutation

    return hilbert_permutation(spec["grid"])


@pytest.mark.parametrize("name", list(SPECS))
def test_block_oracle_matches_full_oracle(name):
    spec = SPECS[name]
    perm = _perm(spec)
    x0, x1, x2 = _inputs(spec)
    full = orc.OracleOperator(perm, spec["text"], spec["text_first"], head_density=spec["density"])
    r0 = full.refresh(0, *x0)
    basis = full.layer(0).basis.clone()
    full.step = 1
    s1 = full.sparse(0, *x1)
    full.step = 2
    r2 = full.refresh(0, *x2)
    v_full = full.drain_validation()

    for qblocks in (None, [0, 2, 5]):
        blk = bo.BlockOracle(perm, spec["text"], spec["text_first"], spec["density"], qblocks=qblocks)
        got_r0 = blk.refresh(*x0, basis=basis)
        blk.step = 1
        got_s1 = blk.sparse(*x1)
        blk.step = 2
        got_r2 = blk.refresh(*x2)
        v_blk = blk.drain_validation()
        for got, ref in ((got_r0, r0), (got_s1, s1), (got_r2, r2)):
            for qb, rows in got.items():
                exp = ref[:, blk.native_rows(qb)]
                cmp = bo.compare_bf16(rows, exp)
                # the same bf16 rounding points; the fp32 / fp64 contractions differ in the
                # last bits, which can move a rounding by one bf16 ulp
                assert cmp["max_abs"] <= 2e-2 or cmp["max_ulps_over_2e-2"] <= 1.0, (qb, cmp)
                assert cmp["mean_rel"] <= 2e-3, (qb, cmp)
        assert torch.equal(blk.state.partition, full.layer(0).partition)
        if qblocks is None:
            assert v_blk[0] == v_full[0]
            assert math.isclose(v_blk[1], v_full[1], rel_tol=1e-3), (v_blk, v_full)
            full_lse = full.layer(0).coarse_lse
            assert float((blk.state.coarse_lse - full_lse).abs().max()) <= 1e-4


def test_sample_qblocks_covers_dense_rows():
    qbs = bo.sample_qblocks(118800, 119056, 8)
    assert qbs[0] == 0 and 927 in qbs
    assert {928, 929, 930} <= set(qbs)  # partial video block shared with text, text blocks
    assert len(qbs) == 8 + 3


@pytest.mark.parametrize("name", list(SPECS))
def test_full_layer_cpu_port_matches_block_oracle(name):
    """The whole-layer CPU port that ``bench.py --impl reference`` times computes the
    same SPARSE step as the oracle, given the same refresh state."""
    from oracle.cpu_baseline import FullLayer

    spec = dict(SPECS[name])
    perm = _perm(spec)
    x0, x1, _ = _inputs(spec)
    blk = bo.BlockOracle(perm, spec["text"], spec["text_first"], spec["density"])
    blk.refresh(*x0)
    blk.step = 1
    exp = blk.sparse(*x1)
    full = FullLayer(spec)
    video = sorted(blk.state.value)
    bf = torch.bfloat16
    for b in range(spec["heads"]):
        st = dict(partition=blk.state.partition[b], basis=blk.state.basis[b], ogl=blk.state.coarse_lse[b],
                  det=torch.cat([blk.state.value[qb][b] for qb in video]) if video else
                  torch.zeros(0, spec["dim"], dtype=torch.float16),
                  dl=torch.cat([blk.state.log_mass[qb][b] for qb in video]) if video else torch.zeros(0))
        got = full.sparse_bank(x1[0][b].to(bf), x1[1][b].to(bf), x1[2][b].to(bf), st)
        for qb, rows in exp.items():
            c = bo.compare_bf16(got[blk.native_rows(qb)], rows[b])
            assert c["max_abs"] <= 2e-2 or c["max_ulps_over_2e-2"] <= 1.0, (b, qb, c)
            assert c["mean_rel"] <= 2e-3, (b, qb, c)
