"""Generate the golden fixtures of tests/golden/ from the REFERENCE implementation.

Run where a checkout of the reference tree exists, named by the environment variable
RECAP_REFERENCE_PATH:  ``RECAP_REFERENCE_PATH=<checkout> python tests/golden/make_golden.py``.

The reference operator (lyraxtg/RECAP ``recap.operator.Operator``) is driven on CPU, fp32,
through its own Python code.  Its GPU-only steps are run as follows:
  * its Triton kernels ``_coarse_tail_kernel``, ``_refresh_detail_kernel`` and
    ``_sparse_merge_kernel`` run unmodified under the Triton interpreter
    (TRITON_INTERPRET=1; fp32 inputs, as the interpreter's bf16 path is unusable), launched
    by the small CPU launchers below in place of their CUDA-only wrappers;
  * the dense refresh uses aten._scaled_dot_product_flash_attention_for_cpu;
  * the external block_sparse_attn head (not in the reference tree) and the two
    closure_stats kernels (which the interpreter cannot run: their bf16 hi/lo dots mix
    dtypes) are replaced by the oracle's restatements - those steps are therefore pinned
    by their definition only.
Each case runs REFRESH, SPARSE (perturbed inputs), and a revalidating REFRESH (perturbed
again), and saves the reference's outputs and bank state.
"""

from __future__ import annotations

import hashlib
import json
import math
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("RECAP_REFERENCE_PATH"):
    raise SystemExit("set RECAP_REFERENCE_PATH to a checkout of the reference tree (lyraxtg/RECAP)")
REF = Path(os.environ["RECAP_REFERENCE_PATH"])
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402

import recap.operator as ref_operator  # noqa: E402
import recap.sparse.attention as ref_attention  # noqa: E402
from recap.config import OperatorConfig  # noqa: E402
from recap.kernels import closure_stats as ref_closure_stats  # noqa: E402
from recap.kernels import coarse_tail as ref_coarse  # noqa: E402
from recap.kernels import detail_cache as ref_detail  # noqa: E402
from recap.sparse.attention import SparseGeometry  # noqa: E402
from recap.sparse.geometry import hilbert_permutation  # noqa: E402
from recap.sparse.layout import Layout  # noqa: E402
from recap.sparse.types import AttentionBranch  # noqa: E402

from oracle import recap_oracle as orc  # noqa: E402


# ----------------------------------------------------------------------------- CPU stand-ins


def head_cpu(query, key, value, kernel_mask):
    """block_sparse_exact on CPU: exact masked attention (oracle restatement)."""
    _, heads, S, d = query.shape
    o, l = orc.masked_attention(query[0].float(), key[0].float(), value[0].float(), kernel_mask.cpu(),
                                1.0 / math.sqrt(d))
    return AttentionBranch(output=o.unsqueeze(0).to(query.dtype), lse=l.unsqueeze(0))


def rotated_moments_cpu(key, key_block_mean, basis, block_counts, *, n_video, block_size, **_):
    var = orc.rotated_variance(key.float(), basis.float(), n_video)
    return key_block_mean.float(), var


def cross_cpu(key, value, key_block_mean, block_counts, *, n_video, block_size, **_):
    return orc.cross_covariance(key.float(), value.float(), key_block_mean.float(), block_counts.float(), n_video)


def coarse_tail_cpu(query, plan, *, scale=None, query_block_size=128, video_query_tokens=None, block_m=32,
                    block_n=32):
    """Launch the reference's _coarse_tail_kernel under the interpreter (CPU tensors)."""
    rows_total = query.shape[-2]
    rows = rows_total if video_query_tokens is None else int(video_query_tokens)
    d = query.shape[-1]
    prefix = query.shape[:-2]
    q = query[..., :rows, :].reshape(-1, rows, d).contiguous()
    nb = plan.key_blocks.shape[-2]
    groups = plan.block_ids.shape[-1]
    qblocks = plan.block_ids.shape[-2]
    if groups == 0:
        return AttentionBranch(output=torch.zeros_like(query),
                               lse=torch.full((*prefix, rows_total), -math.inf))
    qsq = plan.query_square[..., :rows, :].reshape(-1, rows, d).to(q.dtype).contiguous()
    k = plan.key_blocks.reshape(-1, nb, d).to(q.dtype).contiguous()
    v = plan.value_blocks.reshape(-1, nb, d).to(q.dtype).contiguous()
    w = plan.key_variance.reshape(-1, nb, d).to(q.dtype).contiguous()
    counts = plan.block_counts.float().contiguous()
    ids = plan.block_ids.reshape(-1, qblocks, groups).contiguous()
    valid = plan.valid.reshape(-1, qblocks, groups).contiguous()
    bh = q.shape[0]
    out = torch.empty(bh, rows, d, dtype=q.dtype)
    lse = torch.empty(bh, rows)
    gate = torch.empty(bh, rows)
    s = float(scale)
    theta = float(plan.gate_theta)
    ref_coarse._coarse_tail_kernel[(triton.cdiv(rows, block_m), bh)](
        q, qsq, k, w, v, counts, ids, valid, out, lse, gate,
        n_rows=rows, n_groups=groups, n_qblocks=qblocks, d_head=d,
        stride_qh=q.stride(0), stride_qm=q.stride(1), stride_sh=qsq.stride(0), stride_sm=qsq.stride(1),
        stride_kh=k.stride(0), stride_kn=k.stride(1), stride_wh=w.stride(0), stride_wn=w.stride(1),
        stride_vh=v.stride(0), stride_vn=v.stride(1), stride_bh=ids.stride(0), stride_bq=ids.stride(1),
        stride_bg=ids.stride(2), stride_vah=valid.stride(0), stride_vaq=valid.stride(1),
        stride_vag=valid.stride(2), stride_oh=out.stride(0), stride_om=out.stride(1),
        scale=s, half_scale_sq=0.5 * s * s, scale_sq=s * s, theta_sq=theta * theta,
        query_block_size=query_block_size, BLOCK_M=block_m, BLOCK_N=block_n,
        BLOCK_D=triton.next_power_of_2(d),
    )
    drift = plan.value_drift[..., :rows, :].reshape(-1, rows, d).to(q.dtype)
    out = out + gate[..., None].to(q.dtype) * drift
    if rows < rows_total:
        full_out = torch.zeros(bh, rows_total, d, dtype=query.dtype)
        full_lse = torch.full((bh, rows_total), -math.inf)
        full_out[:, :rows] = out
        full_lse[:, :rows] = lse
        out, lse = full_out, full_lse
    return AttentionBranch(output=out.reshape(*prefix, rows_total, d), lse=lse.reshape(*prefix, rows_total))


def refresh_detail_cpu(full_o, full_l, head_o, head_l, coarse_o, coarse_l, permutation, detail, detail_lse, *,
                       video_offset, validation_stats=None, drift_old_lse=None, drift_center=None):
    banks, sequence, dim = full_o.shape
    rows = detail.shape[1]
    ref_detail._refresh_detail_kernel[(triton.cdiv(rows, 32), banks)](
        full_o, full_l, head_o, head_l, coarse_o, coarse_l, permutation, detail, detail_lse,
        detail if validation_stats is None else validation_stats,
        detail if drift_old_lse is None else drift_old_lse,
        detail if drift_center is None else drift_center,
        rows=rows, sequence=sequence, dim=dim, video_offset=int(video_offset),
        stride_fo_b=full_o.stride(0), stride_fo_s=full_o.stride(1), stride_fl_b=full_l.stride(0),
        stride_fl_s=full_l.stride(1), stride_ho_b=head_o.stride(0), stride_ho_s=head_o.stride(1),
        stride_hl_b=head_l.stride(0), stride_hl_s=head_l.stride(1), stride_go_b=coarse_o.stride(0),
        stride_go_s=coarse_o.stride(1), stride_gl_b=coarse_l.stride(0), stride_gl_s=coarse_l.stride(1),
        stride_d_b=detail.stride(0), stride_d_s=detail.stride(1), stride_dl_b=detail_lse.stride(0),
        stride_dl_s=detail_lse.stride(1), BLOCK_M=32, BLOCK_D=triton.next_power_of_2(dim),
        VALIDATE_PREVIOUS=validation_stats is not None, DRIFT_ADMIT=drift_old_lse is not None,
    )


def sparse_merge_cpu(head_output, head_lse, coarse_output, coarse_lse, detail, detail_lse, *, rows,
                     drift_old_lse=None, drift_center=None):
    banks, sequence, dim = head_output.shape
    output = torch.empty_like(head_output)
    ref_detail._sparse_merge_kernel[(triton.cdiv(sequence, 32), banks)](
        head_output, head_lse, coarse_output, coarse_lse, detail, detail_lse,
        detail if drift_old_lse is None else drift_old_lse,
        detail if drift_center is None else drift_center, output,
        rows=int(rows), sequence=sequence, dim=dim,
        stride_ho_b=head_output.stride(0), stride_ho_s=head_output.stride(1), stride_hl_b=head_lse.stride(0),
        stride_hl_s=head_lse.stride(1), stride_go_b=coarse_output.stride(0), stride_go_s=coarse_output.stride(1),
        stride_gl_b=coarse_lse.stride(0), stride_gl_s=coarse_lse.stride(1), stride_d_b=detail.stride(0),
        stride_d_s=detail.stride(1), stride_dl_b=detail_lse.stride(0), stride_dl_s=detail_lse.stride(1),
        stride_o_b=output.stride(0), stride_o_s=output.stride(1), BLOCK_M=32,
        BLOCK_D=triton.next_power_of_2(dim), DRIFT_ADMIT=drift_old_lse is not None,
    )
    return output


def install_stand_ins() -> None:
    ref_operator.block_sparse_exact = head_cpu
    ref_closure_stats.rotated_leaf_moments_triton = rotated_moments_cpu
    ref_closure_stats.pooled_cross_centered_triton_fp32 = cross_cpu
    ref_attention.coarse_tail_attention = coarse_tail_cpu
    ref_detail.refresh_detail = refresh_detail_cpu
    ref_detail.sparse_merge = sparse_merge_cpu


# ----------------------------------------------------------------------------- cases

CASES = {
    # config 1 of the benchmark
    "config1": dict(grid=(8, 16, 16), text=0, text_first=False, heads=2, dim=64, density=0.25, inputs="iid"),
    # text first, partial last video block sharing a kernel block with text
    "textfirst_partial": dict(grid=(3, 12, 20), text=50, text_first=True, heads=2, dim=64, density=0.34,
                              inputs="smooth"),
    # text last, head_dim 128, partial last video block
    "textlast_d128": dict(grid=(4, 9, 14), text=40, text_first=False, heads=2, dim=128, density=0.5,
                          inputs="smooth"),
    # head_dim 128, no text, whole blocks
    "video_d128": dict(grid=(2, 16, 32), text=0, text_first=False, heads=2, dim=128, density=0.25,
                       inputs="smooth"),
}

HILBERT_GRIDS = [(8, 16, 16), (21, 30, 52), (11, 48, 85), (33, 45, 80), (3, 12, 20), (4, 9, 14), (2, 16, 32),
                 (1, 1, 1), (5, 3, 2), (7, 1, 9)]


def case_inputs(spec):
    if spec["inputs"] == "iid":
        return orc.config1_inputs(0)
    return orc.smooth_lowrank(spec["grid"], spec["heads"], spec["dim"], spec["text"], spec["text_first"], seed=0,
                              dtype=torch.float32)


def run_case(name: str, spec: dict) -> dict:
    perm = hilbert_permutation(spec["grid"])
    layout = Layout.from_permutation(perm, text_tokens=spec["text"], text_first=spec["text_first"])
    geometry = SparseGeometry.build(layout, 128)
    cfg = OperatorConfig(head_density=spec["density"])
    op = ref_operator.Operator.build(cfg, geometry, n_layers=1)
    layer, bank = op.layers[0][0], op.banks[0][0]
    q0, k0, v0 = case_inputs(spec)

    def refresh(step, q, k, v):
        op.begin_step(step, ref_operator.REFRESH)
        out, lse = torch.ops.aten._scaled_dot_product_flash_attention_for_cpu(q, k, v, 0.0, False)[:2]
        op._refresh(layer, bank, q, k, v, out, lse)
        return out

    saved = {"spec": spec}
    refresh(0, q0, k0, v0)
    saved["r0_partition"] = bank.partition.clone()
    saved["r0_kernel_mask"] = bank.head_kernel_mask.clone()
    saved["r0_value"] = bank.value.clone()
    saved["r0_log_mass"] = bank.log_mass.clone()
    saved["r0_coarse_lse"] = bank.coarse_lse.clone()
    saved["basis"] = layer._basis.clone()
    q1, k1, v1 = orc.perturb3(q0, k0, v0, seed=1)
    op.begin_step(1, ref_operator.SPARSE)
    saved["s1_out"] = op.attend(0, q1, k1, v1).clone()
    q2, k2, v2 = orc.perturb3(q1, k1, v1, seed=2)
    refresh(2, q2, k2, v2)
    drained = op.drain_validation()
    saved["r2_validation"] = torch.tensor([float(drained[0]), float(drained[1])])
    saved["r2_partition"] = bank.partition.clone()
    saved["r2_value"] = bank.value.clone()
    saved["r2_log_mass"] = bank.log_mass.clone()
    saved["r2_coarse_lse"] = bank.coarse_lse.clone()
    return saved


def main() -> None:
    install_stand_ins()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    hil = {}
    for grid in HILBERT_GRIDS:
        p = np.ascontiguousarray(hilbert_permutation(grid).astype(np.int64))
        hil["x".join(map(str, grid))] = {"sha256": hashlib.sha256(p.tobytes()).hexdigest(),
                                         "head": p[:64].tolist(), "n": int(p.size)}
    (HERE / "hilbert.json").write_text(json.dumps(hil, indent=1))
    for name, spec in CASES.items():
        saved = run_case(name, spec)
        torch.save(saved, HERE / f"{name}.pt")
        print(name, {k: tuple(v.shape) for k, v in saved.items() if torch.is_tensor(v)})


if __name__ == "__main__":
    main()
