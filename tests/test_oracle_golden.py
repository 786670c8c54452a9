"""The CPU oracle against the golden fixtures produced by the reference implementation
(tests/golden/make_golden.py), and the product's host-side Hilbert order against the
reference's permutations."""

import hashlib
import json

import numpy as np
import pytest
import torch

from oracle import recap_oracle as orc
from recap_b200.sparse.geometry import hilbert_permutation

CASES = ["config1", "textfirst_partial", "textlast_d128", "video_d128"]


def _sha(p: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(np.asarray(p, dtype=np.int64)).tobytes()).hexdigest()


def test_hilbert_matches_reference(golden_dir):
    table = json.loads((golden_dir / "hilbert.json").read_text())
    for key, rec in table.items():
        grid = tuple(int(x) for x in key.split("x"))
        perm = hilbert_permutation(grid)
        assert perm.size == rec["n"]
        assert perm[:64].tolist() == rec["head"]
        assert _sha(perm) == rec["sha256"], key


@pytest.mark.parametrize("grid", [(8, 16, 16), (3, 12, 20), (4, 9, 14), (5, 3, 2), (7, 1, 9)])
def test_oracle_hilbert_loop_matches(golden_dir, grid):
    table = json.loads((golden_dir / "hilbert.json").read_text())
    assert _sha(orc.hilbert_permutation(grid)) == table["x".join(map(str, grid))]["sha256"]


def _inputs(spec):
    if spec["inputs"] == "iid":
        return orc.config1_inputs(0)
    return orc.smooth_lowrank(spec["grid"], spec["heads"], spec["dim"], spec["text"], spec["text_first"], seed=0,
                              dtype=torch.float32)


@pytest.mark.parametrize("name", CASES)
def test_oracle_operator_matches_reference(golden_dir, name):
    g = torch.load(golden_dir / f"{name}.pt")
    spec = g["spec"]
    perm = hilbert_permutation(spec["grid"])
    op = orc.OracleOperator(perm, spec["text"], spec["text_first"], head_density=spec["density"],
                            dtype=torch.float32)
    q0, k0, v0 = _inputs(spec)
    op.refresh(0, q0[0], k0[0], v0[0])
    st = op.layer(0)
    assert torch.equal(st.partition, g["r0_partition"][0])
    S = q0.shape[-2]
    assert torch.equal(orc.kernel_block_mask(st.partition, S, len(perm)), g["r0_kernel_mask"])
    scale = g["r0_value"].float().abs().max()
    assert (st.value.float() - g["r0_value"].float()).abs().max() <= 2e-3 * max(1.0, float(scale))
    assert (st.log_mass - g["r0_log_mass"]).abs().max() <= 1e-3
    assert (st.coarse_lse - g["r0_coarse_lse"]).abs().max() <= 1e-4
    q1, k1, v1 = orc.perturb3(q0, k0, v0, seed=1)
    op.step = 1
    out = op.sparse(0, q1[0], k1[0], v1[0])
    ref = g["s1_out"][0]
    assert (out - ref).abs().max() <= 1e-3 * max(1.0, float(ref.abs().max()))
    q2, k2, v2 = orc.perturb3(q1, k1, v1, seed=2)
    op.step = 2
    op.refresh(0, q2[0], k2[0], v2[0])
    age, err = op.drain_validation()
    assert age == int(g["r2_validation"][0])
    assert abs(err - float(g["r2_validation"][1])) <= 1e-3 * float(g["r2_validation"][1])
    assert torch.equal(st.partition, g["r2_partition"][0])
    assert (st.value.float() - g["r2_value"].float()).abs().max() <= 2e-3 * max(1.0, float(scale))


def test_topk_tie_rule_lower_index_wins():
    scores = torch.tensor([[1.0, 3.0, 3.0, 3.0, 0.5]])
    m = orc.topk_mask(scores, 2)
    assert m.tolist() == [[False, True, True, False, False]]


def test_keep_blocks_rounds_half_to_even():
    assert orc.keep_blocks(0.25, 16) == 4
    assert orc.keep_blocks(0.1, 929) == 93
    assert orc.keep_blocks(0.5, 5) == 2  # round(2.5) == 2
    assert orc.keep_blocks(0.01, 10) == 1
