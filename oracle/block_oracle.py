"""The operator's REFRESH / SPARSE state machine at full sequence length, evaluated on
chosen query blocks - TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s parity leg use this module, as the checker.  It restates
the same reference steps as ``oracle/recap_oracle.py`` (whose functions it calls where
they are cheap), but the per-row work is done only for a chosen set of query blocks, so
that a HunyuanVideo-720p head (119,056 tokens) is checked in seconds:

* whole-sequence, per bank (done in full): the Hilbert reorder, block pooling, the
  selection (recap/sparse/attention.py:74-94), the closure statistics
  (recap/sparse/attention.py:156-202: per-block variances in the basis, C_vk), and the
  coarse tail's log-mass for EVERY cached row, which the drift centre needs
  (recap/operator.py:148-150: a mean over all rows);
* per chosen query block: the dense rows (recap/operator.py:254-256), the block-sparse
  head over the block's kept key blocks (recap/kernels/block_sparse.py:78-139), the coarse
  output (recap/kernels/coarse_tail.py:36-186, 237-298), the refinement write with its
  validation (recap/kernels/detail_cache.py:26-186) and the corrected merge
  (recap/kernels/detail_cache.py:188-301).

The refinement bank is therefore held for the chosen rows only, and the validation sums
cover the chosen rows only; with ``qblocks=None`` every query block is chosen and the
sums are the reference's over the whole layer.  The large contractions (Q K^T over the
whole sequence, P V) run in fp32 on the CPU; their rounding (~1e-6 relative) is far below
the bf16 rounding points the comparison tolerates.  The coarse tail follows
``recap_oracle.coarse_tail`` (fp64 with the reference's bf16 rounding points).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import recap_oracle as orc

BLOCK = 128

# Coarse-tail rows that any two implementations may legitimately compute differently
# (recap/kernels/coarse_tail.py:36-186).  The gated quadratic term s^2 qsq.w / 2 is built
# from bf16 operands that each side rounds on its own way there: q.U and the per-block
# variances w are fp32 sums rounded to bf16, and a value near a bf16 midpoint may round
# either way, moving that operand by up to 2^-8 relative.  Such a flip shifts a gated
# block's logit by up to about 0.02 nats and, for a gate within about 1% of its threshold
# (s^2 qsq.w <= theta^2), may switch the gate (a step of up to theta^2 / 2 = 2 nats).  A row
# whose coarse LSE differs from this oracle's by more than FLIP_LSE (about one row in ten
# thousand) is therefore held only to a loose bound in the parity tests, as fp ties are
# exempt in the top-k; NEAR_GATE is the margin reported as a likely gate switch.
NEAR_GATE = 1e-2
FLIP_LSE = 5e-4


def _rd(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return x.to(dtype).float() if dtype != torch.float32 else x.float()


def attention_rows(q_rows: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cols: torch.Tensor | None,
                   scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact softmax attention of ``q_rows`` [m, d] over key columns ``cols`` (None: all),
    fp32 contractions, row sums in fp64; returns (O fp32 [m, d], natural-log LSE [m])."""
    kk = k if cols is None else k.index_select(0, cols)
    vv = v if cols is None else v.index_select(0, cols)
    s = (q_rows @ kk.T) * scale
    m = s.max(-1, keepdim=True).values
    p = torch.exp(s - m)
    l = p.sum(-1, keepdim=True, dtype=torch.float64)
    o = (p @ vv).double() / l
    return o.float(), (m.double() + torch.log(l)).squeeze(-1).float()


def block_columns(kmask_row: torch.Tensor, S: int) -> torch.Tensor:
    """Token indices of the key blocks set in one row of the kernel block mask."""
    blocks = torch.nonzero(kmask_row).flatten().tolist()
    return torch.cat([torch.arange(j * BLOCK, min(S, (j + 1) * BLOCK)) for j in blocks])


@dataclass
class BankState:
    """One layer's detail bank, restricted to the chosen rows."""

    partition: torch.Tensor | None = None        # [banks, nB, nB] bool
    basis: torch.Tensor | None = None            # [banks, d, d]
    value: dict = field(default_factory=dict)    # qb -> [banks, 128, d] fp16
    log_mass: dict = field(default_factory=dict)  # qb -> [banks, 128]
    coarse_lse: torch.Tensor | None = None       # [banks, rows], every cached row
    valid: bool = False
    refreshed_at: int = 0
    pending: tuple | None = None                 # (age, [sum err^2, sum ref^2]) over the chosen rows


class BlockOracle:
    """recap/operator.py:331-527 for one layer of ``banks`` = batch x heads banks, with the
    per-row work restricted to ``qblocks`` (reordered query-block indices; None = all).

    Inputs are ``[banks, S, d]`` fp32 tensors holding model-dtype (bf16) values in the
    model's native token order.  ``basis`` (``[banks, d, d]``) replaces the eigenbasis of
    the first call, as the GPU tests do: ``eigh`` leaves the signs and the rotation inside
    near-degenerate eigenspaces open, and the operator's choice is the one to check the
    rest against."""

    def __init__(self, permutation: np.ndarray, text_tokens: int, text_first: bool, head_density: float,
                 qblocks=None, theta: float = 2.0, rank: int = 4, min_overlap: float = 0.95,
                 dtype: torch.dtype = torch.bfloat16):
        self.perm = np.asarray(permutation)
        self.nv = len(self.perm)
        self.text = int(text_tokens)
        self.text_first = bool(text_first)
        self.S = self.nv + self.text
        self.nB = (self.nv + BLOCK - 1) // BLOCK
        self.NB = (self.S + BLOCK - 1) // BLOCK
        self.rows = (self.nv // BLOCK) * BLOCK
        shared = self.nv % BLOCK != 0 and self.S > self.nv
        self.dense_start = self.nB - 1 if shared else self.nB
        self.density = float(head_density)
        self.theta = float(theta)
        self.rank = int(rank)
        self.min_overlap = float(min_overlap)
        self.dtype = dtype
        self.fwd, self.inv = orc.gather_indices(torch.as_tensor(self.perm), self.text, self.text_first)
        qbs = range(self.NB) if qblocks is None else qblocks
        self.qblocks = sorted({int(b) for b in qbs if 0 <= int(b) < self.NB})
        self.state = BankState()
        self.step = 0
        self.trace: dict = {}
        # per (bank, cached row): the smallest relative margin |s^2 qsq.w - theta^2| / theta^2
        # of any omitted block's gate, over the coarse evaluations of the last call
        self.gate_margin: torch.Tensor | None = None

    # -- helpers --------------------------------------------------------------------------

    def native_rows(self, qb: int) -> torch.Tensor:
        """Native positions of the rows of reordered query block ``qb``."""
        return self.fwd[qb * BLOCK: min(self.S, (qb + 1) * BLOCK)]

    def _reorder(self, x):
        return x[:, self.fwd]

    def _context(self, q_r, k_r, v_r, basis, scale):
        nv = self.nv
        km, counts = orc.pool_blocks(k_r, nv)
        vm, _ = orc.pool_blocks(v_r, nv)
        st = self.state
        if st.basis is None:
            if basis is not None:
                st.basis = basis.float()
            else:
                b0 = orc.closure_basis(orc.within_block_scatter(k_r, km, counts, nv))
                var0 = orc.rotated_variance(k_r, b0, nv)
                st.basis, _ = orc.order_basis(b0, var0, counts)
        var = orc.fold_rank(orc.rotated_variance(k_r, st.basis, nv), self.rank)
        cvk = orc.cross_covariance(k_r, v_r, km, counts, nv)
        qsq = orc.rotated_query_square(q_r[:, :self.rows], st.basis, self.dtype)  # cached rows
        dt = self.dtype
        return dict(km=km, counts=counts, cvk=cvk, qsq=qsq, kb=_rd(km, dt).double(), vb=_rd(vm, dt).double(),
                    wb=_rd(var, dt).double(), logn=torch.log(counts.float()).double(), basis=st.basis)

    def _coarse_bank(self, b, ctx, q_r, partition, scale, rows_sel=None, drift=None):
        """Coarse tail of bank ``b`` (recap/kernels/coarse_tail.py:36-186, 237-298, the
        gated logits of ``recap_oracle.coarse_tail``): LSE over every cached row and, for
        ``rows_sel`` (a list of query blocks), the output rows.  Returns
        (lse [rows], {qb: out [128, d]}, gate margin [rows])."""
        dt = self.dtype
        kb, wb, vb, logn = ctx["kb"][b], ctx["wb"][b], ctx["vb"][b], ctx["logn"]
        s2 = scale * scale
        th2 = self.theta * self.theta
        lse = torch.full((self.rows,), -math.inf, dtype=torch.float32)
        margin = torch.full((self.rows,), math.inf, dtype=torch.float64)
        outs = {}
        want = set(rows_sel or [])
        chunk = 32  # query blocks per chunk
        nqb = self.rows // BLOCK
        for c0 in range(0, nqb, chunk):
            c1 = min(nqb, c0 + chunk)
            r0, r1 = c0 * BLOCK, c1 * BLOCK
            q = _rd(q_r[b, r0:r1], dt).double()
            qs = _rd(ctx["qsq"][b, r0:r1], dt).double()
            s = (q @ kb.T).float().double() * scale + logn
            quad = (qs @ wb.T).float().double()
            gate = quad * s2 <= self.theta * self.theta
            s = s + torch.where(gate, quad * (0.5 * s2), torch.zeros_like(quad))
            omitted = (~partition[b, c0:c1]).repeat_interleave(BLOCK, dim=0)
            margin[r0:r1] = ((quad * s2 - th2).abs() / th2).masked_fill(~omitted, math.inf).min(-1).values
            s = s.masked_fill(~omitted, -math.inf)
            m = s.max(-1, keepdim=True).values
            has = torch.isfinite(m)
            m_safe = torch.where(has, m, torch.zeros_like(m))
            p = torch.exp(s - m_safe)
            l = p.sum(-1, keepdim=True)
            lse[r0:r1] = torch.where(has, m_safe + torch.log(l), torch.full_like(m, -math.inf)).squeeze(-1).float()
            for qb in range(c0, c1):
                if qb not in want:
                    continue
                a, z = (qb - c0) * BLOCK, (qb - c0 + 1) * BLOCK
                if not bool(has[a:z].all()):
                    outs[qb] = torch.zeros(BLOCK, q.shape[1])
                    continue
                pl = p[a:z]
                ll = l[a:z]
                g = (pl * gate[a:z]).sum(-1, keepdim=True) / ll
                o = _rd(((_rd(pl.float(), dt).double() @ vb) / ll).float(), dt)
                gd = _rd(_rd(g.float(), dt) * drift[qb].float(), dt)
                outs[qb] = _rd(o + gd, dt)
        return lse, outs, margin

    def _note_margin(self, margin: torch.Tensor) -> None:
        """Gate margins of the call's coarse tail (the evaluation that defines its coarse LSE)."""
        self.trace["gate_margin"] = margin
        self.gate_margin = margin

    def gate_flips(self, gpu_lse: torch.Tensor) -> tuple[torch.Tensor, int]:
        """Rows of the last call whose coarse LSE (the operator's ``gpu_lse`` [banks, rows]
        against this oracle's) differs by more than FLIP_LSE: (flags [banks, rows], how many
        of them have a gate within NEAR_GATE of its threshold)."""
        mine = self.trace["coarse_lse"].float()
        theirs = gpu_lse.float()
        same_inf = torch.isinf(theirs) & (theirs == mine)
        flip = ((theirs - mine).abs() > FLIP_LSE) & ~same_inf
        return flip, int((flip & (self.trace["gate_margin"] < NEAR_GATE)).sum())

    def _drift_rows(self, ctx, q_r, b, qb, scale):
        q = q_r[b:b + 1, qb * BLOCK:(qb + 1) * BLOCK]
        return orc.value_drift(q, ctx["cvk"][b:b + 1], scale, self.dtype)[0]

    def _kernel_mask(self, partition):
        return orc.kernel_block_mask(partition, self.S, self.nv)

    def _head_rows(self, q_r, k_r, v_r, kmask, b, qb, scale):
        r0, r1 = qb * BLOCK, min(self.S, (qb + 1) * BLOCK)
        cols = block_columns(kmask[b, qb], self.S)
        o, l = attention_rows(q_r[b, r0:r1], k_r[b], v_r[b], cols, scale)
        return _rd(o, self.dtype), l

    def _dense_rows(self, q_r, k_r, v_r, b, qb, scale):
        r0, r1 = qb * BLOCK, min(self.S, (qb + 1) * BLOCK)
        o, l = attention_rows(q_r[b, r0:r1], k_r[b], v_r[b], None, scale)
        return _rd(o, self.dtype), l

    def _video_blocks(self):
        return [qb for qb in self.qblocks if (qb + 1) * BLOCK <= self.rows]

    # -- REFRESH --------------------------------------------------------------------------

    def refresh(self, q, k, v, basis: torch.Tensor | None = None, decision: bool | None = None,
                partition: torch.Tensor | None = None, new_partition: torch.Tensor | None = None) -> dict:
        """recap/operator.py:253-258, 331-473.  Returns {qb: dense output rows [banks, m, d]}.
        ``decision`` (keep the old partition?) replaces the overlap test over these banks
        when the layer spans more banks than the oracle holds.  ``partition`` (first
        refresh) and ``new_partition`` (re-selection) replace this oracle's selection with
        the operator's, once a caller has checked the two agree up to fp ties, so that a
        tie does not change every comparison after it."""
        dt = self.dtype
        q, k, v = (_rd(t, dt) for t in (q, k, v))
        banks, _, d = q.shape
        scale = 1.0 / math.sqrt(d)
        st = self.state
        self.trace = {}
        q_r, k_r, v_r = self._reorder(q), self._reorder(k), self._reorder(v)
        revalidating = st.valid
        if not revalidating:
            st.partition = (orc.head_partition(q_r, k_r, scale, self.density, self.nv) if partition is None
                            else partition.clone())
        ctx = self._context(q_r, k_r, v_r, basis, scale)
        video = self._video_blocks()
        dense = {}
        for qb in self.qblocks:
            dense[qb] = [self._dense_rows(q_r, k_r, v_r, b, qb, scale) for b in range(banks)]

        def write(partition, validate_with=None):
            kmask = self._kernel_mask(partition)
            lse_all = torch.empty(banks, self.rows)
            margin = torch.empty(banks, self.rows, dtype=torch.float64)
            values, masses, dens = {}, {}, {}
            err = torch.zeros(2, dtype=torch.float64)
            center = None
            per_bank = []
            for b in range(banks):
                drift = {qb: self._drift_rows(ctx, q_r, b, qb, scale) for qb in video}
                lse_b, outs, margin[b] = self._coarse_bank(b, ctx, q_r, partition, scale, video, drift)
                lse_all[b] = lse_b
                per_bank.append(outs)
            self._note_margin(margin)
            if validate_with is not None:
                center = orc.drift_center(lse_all, validate_with)
            for qb in video:
                r0, r1 = qb * BLOCK, (qb + 1) * BLOCK
                det_b, dl_b, den_b = [], [], []
                for b in range(banks):
                    oh, lh = self._head_rows(q_r, k_r, v_r, kmask, b, qb, scale)
                    of, lf = dense[qb][b]
                    go = per_bank[b][qb]
                    gl = lse_all[b, r0:r1]
                    args = dict(old_det=None, old_dl=None, old_lse=None, center=None)
                    if validate_with is not None:
                        args = dict(old_det=st.value[qb][b:b + 1].float(), old_dl=st.log_mass[qb][b:b + 1],
                                    old_lse=validate_with[b:b + 1, r0:r1], center=center[b:b + 1])
                    det, dl, stats = _refresh_rows(of[None], lf[None], oh[None], lh[None], go[None], gl[None], **args)
                    if stats is not None:
                        err += stats
                    det_b.append(det[0])
                    dl_b.append(dl[0])
                    # the tail's share of the dense mass, 1 - ratio (the refinement's weight)
                    den_b.append(1.0 - torch.clamp(torch.exp(torch.clamp(lh - lf, max=0.0)), max=1.0 - 1e-6))
                values[qb] = torch.stack(det_b)
                masses[qb] = torch.stack(dl_b)
                dens[qb] = torch.stack(den_b).float()
            self.trace["den"] = dens
            return lse_all, values, masses, (err if validate_with is not None else None), center

        old_lse = st.coarse_lse if revalidating else None
        lse_all, values, masses, stats, center = write(st.partition, old_lse)
        self.trace.update(center=center, coarse_lse=lse_all)
        st.value, st.log_mass = values, masses
        if stats is not None:
            st.pending = (self.step - st.refreshed_at, stats)
        if revalidating:
            new = orc.head_partition(q_r, k_r, scale, self.density, self.nv)
            kept = int((new & st.partition).sum())
            total = max(int(new.sum()), 1)
            self.trace["overlap"] = (kept, total)
            keep = (kept / total >= self.min_overlap) if decision is None else bool(decision)
            if not keep:
                st.partition = new if new_partition is None else new_partition.clone()
                lse_all, values, masses, _, _ = write(st.partition, None)
                st.value, st.log_mass = values, masses
                self.trace["coarse_lse"] = lse_all
        st.coarse_lse = lse_all
        st.refreshed_at = self.step
        st.valid = True
        return {qb: torch.stack([dense[qb][b][0] for b in range(banks)]) for qb in self.qblocks}

    # -- SPARSE ---------------------------------------------------------------------------

    def sparse(self, q, k, v) -> dict:
        """recap/operator.py:478-527.  Returns {qb: output rows [banks, m, d]} (model dtype
        values; the rows of query block qb sit at ``native_rows(qb)`` of the output)."""
        st = self.state
        if not st.valid:
            raise RuntimeError("a sparse call was requested before an exact refresh")
        dt = self.dtype
        q, k, v = (_rd(t, dt) for t in (q, k, v))
        banks, _, d = q.shape
        scale = 1.0 / math.sqrt(d)
        self.trace = {}
        q_r, k_r, v_r = self._reorder(q), self._reorder(k), self._reorder(v)
        ctx = self._context(q_r, k_r, v_r, None, scale)
        kmask = self._kernel_mask(st.partition)
        video = self._video_blocks()
        lse_all = torch.empty(banks, self.rows)
        margin = torch.empty(banks, self.rows, dtype=torch.float64)
        coarse = []
        for b in range(banks):
            drift = {qb: self._drift_rows(ctx, q_r, b, qb, scale) for qb in video}
            lse_b, outs, margin[b] = self._coarse_bank(b, ctx, q_r, st.partition, scale, video, drift)
            lse_all[b] = lse_b
            coarse.append(outs)
        self._note_margin(margin)
        center = orc.drift_center(lse_all, st.coarse_lse)
        self.trace.update(center=center, coarse_lse=lse_all)
        out = {}
        for qb in self.qblocks:
            rows_b = []
            for b in range(banks):
                oh, lh = self._head_rows(q_r, k_r, v_r, kmask, b, qb, scale)
                if qb in video:
                    r0, r1 = qb * BLOCK, (qb + 1) * BLOCK
                    merged = orc.sparse_merge(
                        oh[None], lh[None], coarse[b][qb][None], lse_all[b:b + 1, r0:r1],
                        st.value[qb][b:b + 1].float(), st.log_mass[qb][b:b + 1], BLOCK,
                        st.coarse_lse[b:b + 1, r0:r1], center[b:b + 1])[0]
                    rows_b.append(_rd(merged, dt))
                else:
                    rows_b.append(oh)
            out[qb] = torch.stack(rows_b)
        return out

    def drain_validation(self):
        """(age, sqrt(sum err^2 / sum ref^2)) over the chosen rows (recap/operator.py:531-547)."""
        p = self.state.pending
        self.state.pending = None
        if p is None:
            return None
        age, (num, den) = p
        return age, (math.sqrt(float(num) / float(den)) if float(den) > 0 else float("inf"))


def _refresh_rows(of, lf, oh, lh, go, gl, old_det=None, old_dl=None, old_lse=None, center=None):
    """recap/kernels/detail_cache.py:26-186 for rows already in reordered order (the dense
    rows were computed for the reordered rows, so no permutation is applied here)."""
    of, lf, oh, lh, go, gl = (t.double() for t in (of, lf, oh, lh, go, gl))
    ratio = torch.clamp(torch.exp(torch.clamp(lh - lf, max=0.0)), max=1.0 - 1e-6)
    den = 1.0 - ratio
    stats = None
    if old_det is not None:
        tail_o, tail_l = orc._tail(go, gl, old_det.double(), old_dl.double(),
                                   None if old_lse is None else old_lse.double(),
                                   None if center is None else center.double())
        c = torch.maximum(lh, tail_l)
        wh = torch.exp(lh - c)
        wt = torch.exp(tail_l - c)
        md = torch.clamp(wh + wt, min=1e-30)
        old = (oh * wh[..., None] + tail_o * wt[..., None]) / md[..., None]
        stats = torch.tensor([float(((old - of) ** 2).sum()), float((of ** 2).sum())], dtype=torch.float64)
    tail = (of - ratio[..., None] * oh) / den[..., None]
    det = torch.clamp(tail - go, -6e4, 6e4)
    det = torch.where((ratio > 1 - 1e-3)[..., None], torch.zeros_like(det), det)
    dl = torch.clamp(lf + torch.log(den) - gl, -30.0, 30.0)
    return det.to(torch.float16), dl.float(), stats


def sample_qblocks(n_video: int, seq: int, n_video_blocks: int, seed: int = 0) -> list[int]:
    """Evenly spread cached video query blocks (first and last included) plus every dense
    query block (text rows and a partial video block shared with text)."""
    rows = (n_video // BLOCK) * BLOCK
    nq = rows // BLOCK
    NB = (seq + BLOCK - 1) // BLOCK
    picks = set(np.linspace(0, max(nq - 1, 0), max(1, min(n_video_blocks, nq))).round().astype(int).tolist())
    picks.update(range(nq, NB))  # partial video block and text blocks
    return sorted(picks)


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """One bf16 ulp at magnitude |x| (2^(floor(log2 |x|) - 7))."""
    m = x.abs().float()
    return torch.where(m > 0, torch.exp2(torch.floor(torch.log2(m.clamp_min(1e-30))) - 7), torch.zeros_like(m))


def chain_bound(exp_rows: torch.Tensor, ulps: float) -> torch.Tensor:
    """Elementwise bound for outputs assembled from bf16-rounded values: max(2e-2, ``ulps``
    bf16 ulps of the largest magnitude in the element's row).  ``exp_rows`` [..., rows, d]."""
    row_max = exp_rows.float().abs().amax(-1, keepdim=True)
    return torch.clamp(ulps * bf16_ulp(row_max), min=2e-2).expand_as(exp_rows)


def compare_bf16(got: torch.Tensor, exp: torch.Tensor) -> dict:
    """Elementwise comparison of two tensors of bf16 values: max-abs, mean-rel, and how the
    elements beyond 2e-2 stand against one bf16 ulp of their magnitude (adjacent bf16
    values differ by one ulp: 2^-5 for magnitudes in [4, 8))."""
    got = got.float()
    exp = exp.float()
    diff = (got - exp).abs()
    mag = torch.maximum(got.abs(), exp.abs())
    ulp = torch.where(mag > 0, torch.exp2(torch.floor(torch.log2(mag.clamp_min(1e-30))) - 7), torch.zeros_like(mag))
    over = diff > 2e-2
    return {
        "max_abs": float(diff.max()) if diff.numel() else 0.0,
        "mean_rel": float(diff.mean() / exp.abs().mean().clamp_min(1e-30)) if diff.numel() else 0.0,
        "n": int(diff.numel()),
        "n_over_2e-2": int(over.sum()),
        "max_ulps_over_2e-2": float((diff[over] / ulp[over]).max()) if bool(over.any()) else 0.0,
        "max_abs_ref": float(exp.abs().max()) if diff.numel() else 0.0,
    }


def selection_mismatches(got: torch.Tensor, q_r: torch.Tensor, k_r: torch.Tensor, head_density: float,
                         n_video: int) -> int:
    """Selected blocks that differ from the oracle's top-k beyond fp ties: a differing block
    is accepted only where its score is within 4 fp32 ulp of the k-th score of its row
    (torch.topk leaves the order of equal scores open; the operator takes lower indices
    first).  The forced partial row and column (recap/sparse/attention.py:88-94) must match
    exactly.  ``got`` [banks, nB, nB] bool; q_r, k_r [banks, S, d] reordered."""
    d = q_r.shape[-1]
    qm, _ = orc.pool_blocks(q_r, n_video)
    km, _ = orc.pool_blocks(k_r, n_video)
    scores = orc.block_scores(qm, km, 1.0 / math.sqrt(d))
    keep = orc.keep_blocks(head_density, qm.shape[-2])
    ref = orc.topk_mask(scores, keep)
    srt = torch.sort(scores.double(), dim=-1, descending=True).values
    kth = srt[..., keep - 1: keep]
    tol = 4 * torch.finfo(torch.float32).eps * kth.abs().clamp_min(1e-30)
    tie = (scores.double() - kth).abs() <= tol
    if n_video % BLOCK:
        ref[..., -1, :] = True
        ref[..., :, -1] = True
        tie[..., -1, :] = False
        tie[..., :, -1] = False
    diff = got.bool() != ref
    return int((diff & ~tie).sum())
