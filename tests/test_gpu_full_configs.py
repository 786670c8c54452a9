"""Operator parity at the benchmark's own sequence lengths: BASELINE configs 2 (Wan2.1,
32,760 video tokens, partial block 255), 3 (CogVideoX, 226 text tokens first, d = 64,
guidance batched as batch 2 like recap/models/cogvideox.py:17) and 4 (HunyuanVideo 720p,
119,056 tokens, text last), each on a 2-head slice, through
REFRESH -> SPARSE -> revalidating REFRESH -> SPARSE of ``recap_b200.Operator.attend``.

The checker is the block oracle (oracle/block_oracle.py): the whole-sequence work in full
(selection, closure statistics, the coarse log-mass of every cached row for the drift
centre) and the per-row work on chosen query blocks - every block for config 2, spread
video blocks plus every dense (text and partial) block for configs 3 and 4.

Tolerances (the benchmark's parity criteria, max-abs 2e-2 and mean-rel 1e-2):
* REFRESH outputs (dense attention) within max-abs 2e-2 or one bf16 ulp of the row's
  largest magnitude;
* SPARSE outputs within max-abs 2e-2 or three bf16 ulps of the row's largest magnitude.
  The corrected output carries three values the reference rounds to bf16: the dense
  output and the head output at the refresh, whose difference the refinement stores
  divided by the tail's share of the mass (1 - ratio, as small as 1e-3), and the head
  output at the step.  Each may land on a neighbouring bf16 value in any two
  implementations; the merge multiplies the refinement by the tail's share at the step,
  so each such rounding reaches the output as about one ulp of the rounded values'
  magnitude (three ulps are 0.0234 for magnitudes in [1, 2)).  The count of elements over
  2e-2 is printed (a handful per million);
* mean-rel 1e-2 over every checked element;
* selected blocks bit-exact except documented fp ties; the coarse LSE of every cached row
  within 5e-3; the validation error e_detail (config 2, every row) within 2e-2 relative.
Two tie rules: a top-k selection within 4 fp32 ulp of a row's k-th score, and the coarse
tail's bf16 operand roundings (oracle/block_oracle.py FLIP_LSE): a row whose coarse LSE -
the operator's, recomputed through the same deterministic kernels for a SPARSE call -
differs from the oracle's by more than 5e-4 (at most one row in two thousand; about one in
ten thousand observed) is held to max-abs 0.1 instead of the elementwise bounds in the step
that used it, and still counts in the means; the coarse LSE of every cached row is bounded
(max 0.25, mean 2e-4, 99.9th percentile 2e-3).  Every case prints its achieved figures, the
exempt rows and their largest output difference."""

import math

import pytest
import torch

from oracle import block_oracle as bo
from oracle import recap_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"

CONFIGS = {
    "wan_config2": dict(grid=(21, 30, 52), text=0, text_first=False, heads=12, dim=128, density=0.2, batch=1,
                        video_blocks=None),
    # step 2 on unrelated inputs (another seed): the revalidating refresh re-selects
    "wan_config2_rerank": dict(grid=(21, 30, 52), text=0, text_first=False, heads=12, dim=128, density=0.2,
                               batch=1, video_blocks=None, fresh_step2=True),
    "cog_config3_batch2": dict(grid=(11, 48, 85), text=226, text_first=True, heads=48, dim=64, density=0.15,
                               batch=2, video_blocks=24),
    "hunyuan_config4": dict(grid=(33, 45, 80), text=256, text_first=False, heads=24, dim=128, density=0.1,
                            batch=1, video_blocks=12),
}
HEADS = 2  # the slice of each layer's heads that is checked
EXEMPT_BOUND = 0.1  # rows whose coarse LSE measurably differs (oracle/block_oracle.py FLIP_LSE)


def _inputs(spec):
    """[batch, 2, S, d] bf16 Q/K/V (heads 0-1 of the layer's seeded generator; batch element
    i from seed 11 i), and the three perturbed sets of the later steps (step 2 from seed 5
    instead when ``fresh_step2``)."""
    bf = torch.bfloat16

    def draw(seed):
        per_batch = [orc.smooth_lowrank(spec["grid"], spec["heads"], spec["dim"], spec["text"], spec["text_first"],
                                        seed=seed + 11 * i, head_slice=slice(0, HEADS), dtype=bf)
                     for i in range(spec["batch"])]
        return tuple(torch.cat([pb[t] for pb in per_batch]).float() for t in range(3))

    xs = [draw(0)]
    for s in (1, 2, 3):
        base = draw(5) if (s == 2 and spec.get("fresh_step2")) else xs[-1]
        xs.append(tuple(t.to(bf).float() for t in orc.perturb3(*base, seed=s)))
    return xs


def _selection_ok(got: torch.Tensor, q_r, k_r, spec, nv) -> int:
    """Number of selections that differ from the oracle beyond fp ties (0 = pass)."""
    return bo.selection_mismatches(got, q_r, k_r, spec["density"], nv)


def _check_rows(tag, got_native, exp_rows, oracle, stats, ulps, exempt=None):
    """Elementwise: every element of a row that is not ``exempt`` ([banks, rows] bool over
    the cached rows: gate flips) within max(2e-2, ``ulps`` bf16 ulps of its row's largest
    magnitude); mean-rel over all rows.  Prints the achieved figures."""
    n_ex = n_over = n_el = 0
    ex_max = 0.0
    for qb, rows in exp_rows.items():
        g = got_native[:, oracle.native_rows(qb)].float()
        e = rows.float()
        r0, r1 = qb * 128, qb * 128 + e.shape[1]
        keep = torch.ones(e.shape[:2], dtype=torch.bool)
        if exempt is not None and r0 < exempt.shape[1]:
            keep = ~exempt[:, r0:min(r1, exempt.shape[1])]
            keep = torch.cat([keep, torch.ones(e.shape[0], e.shape[1] - keep.shape[1], dtype=torch.bool)], 1)
        diff = (g - e).abs()
        n_ex += int((~keep).sum())
        if bool((~keep).any()):
            ex_max = max(ex_max, float(diff[~keep].max()))
            assert ex_max <= EXEMPT_BOUND, f"{tag} block {qb}: a coarse-LSE-flip row differs by {ex_max}"
        over = (diff > bo.chain_bound(e, ulps)) & keep[..., None]
        n_over += int(((diff > 2e-2) & keep[..., None]).sum())
        n_el += diff.numel()
        if bool(over.any()):
            b, r, c = torch.nonzero(over)[0].tolist()
            raise AssertionError(f"{tag} block {qb}: bank {b} row {r} col {c}: got {float(g[b, r, c])}, "
                                 f"expected {float(e[b, r, c])}, row max {float(e[b, r].abs().max())}; "
                                 f"{int(over.sum())} elements over the bound")
    allg = torch.cat([got_native[:, oracle.native_rows(qb)].reshape(-1).float() for qb in exp_rows])
    alle = torch.cat([exp_rows[qb].reshape(-1).float() for qb in exp_rows])
    total = bo.compare_bf16(allg, alle)
    stats[tag] = total
    print(f"{tag}: max_abs {total['max_abs']:.3e} (|ref| <= {total['max_abs_ref']:.2f}), "
          f"mean_rel {total['mean_rel']:.3e}; outside gate-flip rows {n_over} of {n_el} elements over 2e-2 "
          f"(within {ulps} bf16 ulp of their row's magnitude); {n_ex} gate-flip rows, max abs there {ex_max:.3e}")
    assert total["mean_rel"] <= 1e-2, (tag, total)
    return total


def _flips(tag, oracle, gpu_lse):
    """Rows of the call whose coarse LSE differs from the oracle's by more than FLIP_LSE
    (bf16 operand roundings of the gated term, gate switches); the LSE over every cached
    row stays bounded."""
    flip, near = oracle.gate_flips(gpu_lse)
    diff = (gpu_lse - oracle.trace["coarse_lse"]).abs()
    finite = torch.isfinite(diff)
    q999 = float(torch.quantile(diff[finite].double(), 0.999))
    print(f"{tag} coarse LSE over all {diff.numel()} cached rows: {int(flip.sum())} rows over 5e-4 "
          f"({near} with a gate within 1% of its threshold), max {float(diff[finite].max()):.3e}, "
          f"mean {float(diff[finite].mean()):.3e}, 99.9th percentile {q999:.3e}")
    assert int(flip.sum()) <= max(4, diff.numel() // 2000), f"{tag}: {int(flip.sum())} coarse LSE rows over 5e-4"
    # a switched gate moves the LSE by log(1 + p (e^2 - 1)) for a block of tail share p
    assert float(diff[finite].max()) <= 0.25 and float(diff[finite].mean()) <= 2e-4 and q999 <= 2e-3
    return flip


def _gpu_coarse_lse(op, x_dev, partition, old_lse):
    """The operator's coarse LSE of a SPARSE call, recomputed through the same kernels
    (deterministic) for the cached rows."""
    layer = op.layers[0][0]
    q = x_dev[0]
    scale = 1.0 / math.sqrt(q.shape[-1])
    inputs = layer.prepare(*x_dev, q_mean=False)
    ctx = layer.coarse_tail_context(inputs, scale)
    _, gl, _ = layer.coarse_tail_apply(inputs, ctx, partition, scale, old_lse=old_lse,
                                       status=op.status_word(q.device))
    return gl.cpu()


@pytest.mark.parametrize("name", list(CONFIGS))
def test_operator_full_length_parity(name):
    from recap_b200 import REFRESH, SPARSE, Operator, OperatorConfig
    from recap_b200.sparse import Layout, SparseGeometry, hilbert_permutation

    spec = CONFIGS[name]
    perm = hilbert_permutation(spec["grid"])
    layout = Layout.from_permutation(perm, text_tokens=spec["text"], text_first=spec["text_first"])
    op = Operator.build(OperatorConfig(head_density=spec["density"]), SparseGeometry.build(layout, 128), n_layers=1)
    nv = len(perm)
    S = nv + spec["text"]
    B = spec["batch"]
    banks = B * HEADS
    xs = _inputs(spec)
    bf = torch.bfloat16

    def dev(x):
        return [t.reshape(B, HEADS, S, -1).to(bf).to(DEV) for t in x]

    def flat(t):
        return t.reshape(banks, *t.shape[2:])

    gpu = {}
    op.begin_step(0, REFRESH)
    gpu["r0"] = flat(op.attend(0, *dev(xs[0])).float().cpu())
    bank = op.banks[0][0]
    part0 = bank.partition.cpu().reshape(banks, *bank.partition.shape[-2:]).clone()
    value0 = bank.value.cpu().clone()
    mass0 = bank.log_mass.cpu().clone()
    lse0 = bank.coarse_lse.cpu().clone()
    basis = op.layers[0][0].basis.cpu().clone()
    op.begin_step(1, SPARSE)
    gpu["s1"] = flat(op.attend(0, *dev(xs[1])).float().cpu())
    gl1 = _gpu_coarse_lse(op, dev(xs[1]), bank.partition, bank.coarse_lse)
    op.begin_step(2, REFRESH)
    gpu["r2"] = flat(op.attend(0, *dev(xs[2])).float().cpu())
    val2 = op.drain_validation()
    part2 = bank.partition.cpu().reshape(banks, *bank.partition.shape[-2:]).clone()
    lse2 = bank.coarse_lse.cpu().clone()
    op.begin_step(3, SPARSE)
    gpu["s3"] = flat(op.attend(0, *dev(xs[3])).float().cpu())
    gl3 = _gpu_coarse_lse(op, dev(xs[3]), bank.partition, bank.coarse_lse)
    op.check_device_status()

    x = [tuple(flat(t) for t in xi) for xi in xs]
    qblocks = None if spec["video_blocks"] is None else bo.sample_qblocks(nv, S, spec["video_blocks"])
    oracle = bo.BlockOracle(perm, spec["text"], spec["text_first"], spec["density"], qblocks=qblocks)

    # selection: bit-exact except fp ties, then the oracle continues from the operator's
    # partition so that a tie does not change every later comparison
    fwd = oracle.fwd
    q_r0, k_r0 = x[0][0][:, fwd], x[0][1][:, fwd]
    assert _selection_ok(part0, q_r0, k_r0, spec, nv) == 0
    stats = {}

    # REFRESH 0 (first), on the operator's tie-checked partition
    exp = oracle.refresh(*x[0], basis=basis, partition=part0)
    _check_rows("r0", gpu["r0"], exp, oracle, stats, ulps=1)
    flip0 = _flips("r0", oracle, lse0)
    # The refinement value det = (of - ratio oh) / (1 - ratio) - go carries the bf16 roundings
    # of the dense and head outputs divided by the tail's share 1 - ratio (down to 1e-3), so
    # it is compared weighted by that share: the sparse step adds det to the tail, whose
    # weight in the merge is proportional to it (recap/kernels/detail_cache.py:267-292).
    worst = 0.0
    for qb in oracle.state.value:
        r0, r1 = qb * 128, (qb + 1) * 128
        ok = ~flip0[:, r0:r1]
        w = oracle.trace["den"][qb][ok][:, None]
        dv = bo.compare_bf16(value0[:, r0:r1][ok].float() * w, oracle.state.value[qb][ok].float() * w)
        worst = max(worst, dv["mean_rel"])
        assert dv["mean_rel"] <= 2e-2, (qb, dv)
        assert float((mass0[:, r0:r1] - oracle.state.log_mass[qb])[ok].abs().max()) <= 5e-2
    print(f"r0 refinement value (weighted by the tail share): worst block mean_rel {worst:.3e}")

    oracle.step = 1
    exp = oracle.sparse(*x[1])
    flip1 = _flips("s1", oracle, gl1)
    _check_rows("s1", gpu["s1"], exp, oracle, stats, ulps=3, exempt=flip0 | flip1)

    oracle.step = 2
    keep = bool(torch.equal(part2, part0))
    new_part = None if keep else part2
    if not keep:
        assert _selection_ok(part2, x[2][0][:, fwd], x[2][1][:, fwd], spec, nv) == 0
    exp = oracle.refresh(*x[2], decision=keep, new_partition=new_part)
    kept, total = oracle.trace["overlap"]
    print(f"r2 overlap {kept}/{total} = {kept / total:.4f} -> {'keep' if keep else 're-rank'}")
    # the layer-wide decision must be the oracle's unless the overlap sits on the threshold
    if abs(kept / total - 0.95) > 1e-3:
        assert keep == (kept / total >= 0.95)
    _check_rows("r2", gpu["r2"], exp, oracle, stats, ulps=1)
    flip2 = _flips("r2", oracle, lse2)
    if qblocks is None:
        age, err = val2
        rage, rerr = oracle.drain_validation()
        print(f"r2 e_detail {err:.6f} (oracle {rerr:.6f}), age {age}")
        assert age == rage and abs(err - rerr) <= 2e-2 * rerr

    oracle.step = 3
    exp = oracle.sparse(*x[3])
    flip3 = _flips("s3", oracle, gl3)
    _check_rows("s3", gpu["s3"], exp, oracle, stats, ulps=3, exempt=flip2 | flip3)
