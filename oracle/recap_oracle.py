"""CPU oracle of RECAP's corrected sparse attention operator.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this module, and
only as the checker or the timed CPU baseline; the product (``recap_b200``) never calls
it.

A plain torch-CPU restatement of the reference's operator path (lyraxtg/RECAP, files
under ``recap/``), one function per reference step, each citing the lines it follows.
``dtype`` arguments name the model dtype of the reference call (``q.dtype``): wherever
the reference casts or stores in that dtype, the oracle rounds to it, so the same code
serves the fp32 golden runs and the bf16 GPU comparisons.

Pinning: ``tests/golden/make_golden.py`` ran the reference's own Python (and its Triton
kernels under the Triton interpreter) on seeded inputs and saved the outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against them.  The
block-sparse head (``block_sparse_attn``, mit-han-lab Block-Sparse-Attention @ 49d6c39)
is not in the reference tree and has no golden vectors: it is restated as exact masked
softmax attention, so parity of that step is unpinned beyond its mathematical definition.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

BLOCK = 128


def _rd(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Round to the model dtype and back to fp32 (identity for fp32)."""
    return x.to(dtype).float() if dtype != torch.float32 else x.float()


# ----------------------------------------------------------------------------- geometry


def hilbert_permutation(grid) -> np.ndarray:
    """recap/sparse/geometry.py:27-67 - 3-D Hilbert order, x leading, stable argsort.
    Written as a per-token loop over Skilling's transposed-index steps (slow; small grids)."""
    T, H, W = (int(g) for g in grid)
    bits = max(1, math.ceil(math.log2(max(T, H, W))))
    keys = []
    for t in range(T):
        for y in range(H):
            for x in range(W):
                X = [x, y, t]
                q = 1 << (bits - 1)
                while q > 1:
                    p = q - 1
                    for i in range(3):
                        if X[i] & q:
                            X[0] ^= p
                        else:
                            s = (X[0] ^ X[i]) & p
                            X[0] ^= s
                            X[i] ^= s
                    q >>= 1
                for i in range(1, 3):
                    X[i] ^= X[i - 1]
                s = 0
                q = 1 << (bits - 1)
                while q > 1:
                    if X[2] & q:
                        s ^= q - 1
                    q >>= 1
                X = [c ^ s for c in X]
                idx = 0
                for b in range(bits - 1, -1, -1):
                    for i in range(3):
                        idx = (idx << 1) | ((X[i] >> b) & 1)
                keys.append((idx, t * H * W + y * W + x))
    order = sorted(range(len(keys)), key=lambda i: keys[i][0])  # stable
    return np.array([keys[i][1] for i in order], dtype=np.int64)


def gather_indices(permutation: torch.Tensor, text_tokens: int, text_first: bool):
    """recap/sparse/layout.py:48-68 - (reorder, restore) gather indices."""
    p = torch.as_tensor(permutation, dtype=torch.long)
    nv, tt = p.numel(), int(text_tokens)
    inv = torch.argsort(p)
    text = torch.arange(tt)
    if text_first:
        return torch.cat((p + tt, text)), torch.cat((text + nv, inv))
    return torch.cat((p, text + nv)), torch.cat((inv, text + nv))


# ----------------------------------------------------------------------------- selection


def pool_blocks(x: torch.Tensor, n_video: int):
    """recap/sparse/pooling.py:10-34 - block means over the video tokens, fp32 sums."""
    xv = x[..., :n_video, :].float()
    nb = (n_video + BLOCK - 1) // BLOCK
    pad = nb * BLOCK - n_video
    if pad:
        xv = torch.nn.functional.pad(xv, (0, 0, 0, pad))
    counts = torch.full((nb,), float(BLOCK))
    if pad:
        counts[-1] = BLOCK - pad
    s = xv.reshape(*xv.shape[:-2], nb, BLOCK, xv.shape[-1]).sum(-2)
    return s / counts.view(*([1] * (s.dim() - 2)), nb, 1), counts


def block_scores(qm: torch.Tensor, km: torch.Tensor, scale: float) -> torch.Tensor:
    """recap/sparse/router.py:17-18 - fp32 matmul, then the scale."""
    s = torch.matmul(qm.float(), km.float().transpose(-1, -2))
    return s * float(scale)


def topk_mask(scores: torch.Tensor, keep: int) -> torch.Tensor:
    """recap/sparse/router.py:19-22 - top-k per row as a bool mask.  torch.topk leaves the
    order of equal scores unspecified; here lower block indices win (a stable sort)."""
    k = max(1, min(int(keep), scores.shape[-1]))
    order = torch.sort(scores, dim=-1, descending=True, stable=True).indices[..., :k]
    mask = torch.zeros_like(scores, dtype=torch.bool)
    mask.scatter_(-1, order, True)
    return mask


def keep_blocks(head_density: float, n_blocks: int) -> int:
    """recap/sparse/attention.py:84 (Python round: half to even)."""
    return max(1, round(float(head_density) * n_blocks))


def head_partition(q_r: torch.Tensor, k_r: torch.Tensor, scale: float, head_density: float,
                   n_video: int) -> torch.Tensor:
    """recap/sparse/attention.py:74-94 - pool, score, top-k, then a trailing partial video
    block selected in full as a row and as a column."""
    qm, _ = pool_blocks(q_r, n_video)
    km, _ = pool_blocks(k_r, n_video)
    nb = qm.shape[-2]
    mask = topk_mask(block_scores(qm, km, scale), keep_blocks(head_density, nb))
    if n_video % BLOCK:
        mask[..., -1, :] = True
        mask[..., :, -1] = True
    return mask


def kernel_block_mask(video_mask: torch.Tensor, S: int, n_video: int) -> torch.Tensor:
    """recap/kernels/block_sparse.py:52-75."""
    nb = math.ceil(n_video / BLOCK)
    NB = math.ceil(S / BLOCK)
    out = torch.zeros((*video_mask.shape[:-2], NB, NB), dtype=torch.bool)
    out[..., :nb, :nb] = video_mask
    shared = n_video % BLOCK != 0 and S > n_video
    ds = nb - 1 if shared else nb
    out[..., ds:, :] = True
    out[..., :, ds:] = True
    return out


# ----------------------------------------------------------------------------- attention


def masked_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kmask: torch.Tensor | None,
                     scale: float):
    """Exact softmax attention restricted to the kept 128x128 tiles, per bank: the contract
    of block_sparse_attn_func as called at recap/kernels/block_sparse.py:117-139 (O and the
    natural-log LSE).  ``kmask`` None = dense.  q/k/v: [banks, S, d] fp32."""
    banks, S, d = q.shape
    NB = math.ceil(S / BLOCK)
    out = torch.empty(banks, S, d)
    lse = torch.empty(banks, S)
    for b in range(banks):
        for i in range(NB):
            r0, r1 = i * BLOCK, min(S, (i + 1) * BLOCK)
            if kmask is None:
                cols = torch.arange(S)
            else:
                blocks = torch.nonzero(kmask[b, i]).flatten().tolist()
                cols = torch.cat([torch.arange(j * BLOCK, min(S, (j + 1) * BLOCK)) for j in blocks])
            s = (q[b, r0:r1].double() @ k[b, cols].double().T) * scale
            m = s.max(-1, keepdim=True).values
            p = torch.exp(s - m)
            l = p.sum(-1, keepdim=True)
            out[b, r0:r1] = ((p @ v[b, cols].double()) / l).float()
            lse[b, r0:r1] = (m + torch.log(l)).squeeze(-1).float()
    return out, lse


# ----------------------------------------------------------------------------- closure


def within_block_scatter(k_r: torch.Tensor, kmean: torch.Tensor, counts: torch.Tensor, n_video: int):
    """recap/sparse/closure.py:42-73 - pooled within-block key scatter / sum(counts)."""
    banks, _, d = k_r.shape
    nb = kmean.shape[-2]
    kv = k_r[:, :n_video].float()
    pad = nb * BLOCK - n_video
    if pad:
        kv = torch.nn.functional.pad(kv, (0, 0, 0, pad))
    c = kv.reshape(banks, nb, BLOCK, d) - kmean.float().unsqueeze(2)
    if pad:
        c[:, -1, BLOCK - pad:] = 0.0
    c = c.reshape(banks, nb * BLOCK, d)
    return torch.einsum("btd,bte->bde", c, c) / counts.sum()


def closure_basis(scatter: torch.Tensor) -> torch.Tensor:
    """recap/sparse/closure.py:76-81."""
    sym = 0.5 * (scatter + scatter.transpose(-1, -2))
    return torch.linalg.eigh(sym.float())[1]


def rotated_variance(k_r: torch.Tensor, basis: torch.Tensor, n_video: int) -> torch.Tensor:
    """recap/kernels/closure_stats.py:96-189, 242 - per-block population variance of K U,
    two passes (mean of K U, then squared deviations), clamped at 0."""
    banks, _, d = k_r.shape
    nb = math.ceil(n_video / BLOCK)
    out = torch.empty(banks, nb, d)
    for j in range(nb):
        t0, t1 = j * BLOCK, min(n_video, (j + 1) * BLOCK)
        r = torch.bmm(k_r[:, t0:t1].double(), basis.double())
        m = r.mean(1, keepdim=True)
        out[:, j] = ((r - m) ** 2).mean(1).float()
    return out.clamp_min(0.0)


def cross_covariance(k_r: torch.Tensor, v_r: torch.Tensor, kmean: torch.Tensor, counts: torch.Tensor,
                     n_video: int) -> torch.Tensor:
    """recap/kernels/closure_stats.py:27-94, 246-290 - sum_t v_t (k_t - kbar_blk(t))^T / N."""
    banks, _, d = k_r.shape
    kv = k_r[:, :n_video].double()
    blk = torch.arange(n_video) // BLOCK
    c = kv - kmean.double()[:, blk]
    return (torch.einsum("btv,btk->bvk", v_r[:, :n_video].double(), c) / counts.double().sum()).float()


def order_basis(basis: torch.Tensor, variance: torch.Tensor, counts: torch.Tensor):
    """recap/sparse/attention.py:136-152 - columns by descending count-weighted variance."""
    w = counts.reshape(1, -1, 1)
    pooled = (variance.float() * w).sum(1) / w.sum().clamp_min(1.0)
    order = torch.argsort(pooled, dim=-1, descending=True)
    b = torch.gather(basis, 2, order.unsqueeze(1).expand(-1, basis.shape[1], -1))
    v = torch.gather(variance, 2, order.unsqueeze(1).expand(-1, variance.shape[1], -1))
    return b.contiguous(), v.contiguous()


def fold_rank(variance: torch.Tensor, rank: int) -> torch.Tensor:
    """recap/sparse/closure.py:96-104."""
    d = variance.shape[-1]
    if rank <= 0 or rank >= d:
        return variance
    tail = variance[..., rank:].sum(-1, keepdim=True) / float(d - rank)
    return torch.cat([variance[..., :rank], tail.expand(*variance.shape[:-1], d - rank)], -1)


def rotated_query_square(q_video: torch.Tensor, basis: torch.Tensor, dtype) -> torch.Tensor:
    """recap/sparse/closure.py:84-86 - bmm in the model dtype, squared in it."""
    x = _rd(torch.bmm(_rd(q_video, dtype).double(), _rd(basis, dtype).double()).float(), dtype)
    return _rd(x * x, dtype)


def value_drift(q_video: torch.Tensor, cvk: torch.Tensor, scale: float, dtype) -> torch.Tensor:
    """recap/sparse/closure.py:89-93 - scale * bmm(q, C^T) in the model dtype."""
    x = _rd(torch.bmm(_rd(q_video, dtype).double(), _rd(cvk, dtype).double().transpose(-1, -2)).float(), dtype)
    return _rd(float(scale) * x, dtype)


# ----------------------------------------------------------------------------- coarse tail


def coarse_tail(q_r: torch.Tensor, kmean: torch.Tensor, vmean: torch.Tensor, variance: torch.Tensor,
                counts: torch.Tensor, partition: torch.Tensor, qsq: torch.Tensor, drift: torch.Tensor,
                scale: float, theta: float, rows: int, dtype):
    """recap/kernels/coarse_tail.py:36-186 and 237-298, recap/sparse/planner.py:24-27,
    recap/sparse/attention.py:229-231.  q_r [banks, S, d]; partition [banks, nB, nB];
    returns (out [banks, rows, d] fp32 holding model-dtype values, lse [banks, rows]).
    The softmax is taken in one pass with the exact row maximum (the kernel's online form
    with 32-wide tiles differs only in where P is rounded)."""
    banks, _, d = q_r.shape
    nb = kmean.shape[-2]
    k = _rd(kmean, dtype).double()
    v = _rd(vmean, dtype).double()
    w = _rd(variance, dtype).double()
    logn = torch.log(counts.float()).double()
    out = torch.zeros(banks, rows, d)
    lse = torch.full((banks, rows), -math.inf)
    for b in range(banks):
        for qb in range(rows // BLOCK):
            r0, r1 = qb * BLOCK, (qb + 1) * BLOCK
            omitted = ~partition[b, qb]
            if not bool(omitted.any()):
                continue
            q = _rd(q_r[b, r0:r1], dtype).double()
            qs = _rd(qsq[b, r0:r1], dtype).double()
            s = (q @ k[b].T).float().double() * scale + logn
            quad = (qs @ w[b].T).float().double()
            gate = quad * (scale * scale) <= theta * theta
            s = s + torch.where(gate, quad * (0.5 * scale * scale), torch.zeros_like(quad))
            s[:, ~omitted] = -math.inf
            m = s.max(-1, keepdim=True).values
            p = torch.exp(s - m)
            l = p.sum(-1, keepdim=True)
            g = (p * gate).sum(-1, keepdim=True) / l
            o = (_rd(p.float(), dtype).double() @ v[b]) / l
            o = _rd(o.float(), dtype)
            gd = _rd(_rd(g.float(), dtype) * drift[b, r0:r1].float(), dtype)
            out[b, r0:r1] = _rd(o + gd, dtype)
            lse[b, r0:r1] = (m + torch.log(l)).squeeze(-1).float()
    return out, lse


def drift_center(coarse_lse: torch.Tensor, old_lse: torch.Tensor) -> torch.Tensor:
    """recap/operator.py:148-150."""
    return (coarse_lse - old_lse).mean(dim=1)


# ----------------------------------------------------------------------------- merge/refresh


def _tail(go, gl, det, dl, old_lse, center):
    """The drift-weighted tail (recap/kernels/detail_cache.py:267-287)."""
    if old_lse is None:
        return go + det, gl + dl
    admit = torch.exp(-torch.abs(gl - old_lse - center[:, None]))
    cl = gl + dl
    tc = torch.maximum(gl, cl)
    ms = (1 - admit) * torch.exp(gl - tc)
    mc = admit * torch.exp(cl - tc)
    den = torch.clamp(ms + mc, min=1e-30)
    return (go * ms[..., None] + (go + det) * mc[..., None]) / den[..., None], tc + torch.log(den)


def sparse_merge(head_o, head_lse, go, gl, det, dl, rows, old_lse=None, center=None):
    """recap/kernels/detail_cache.py:188-301, 402-456.  head_o [banks, S, d] (model-dtype
    values), go/det [banks, rows, d]; returns fp32 [banks, S, d] before the output cast."""
    out = head_o.float().clone()
    oh = head_o[:, :rows].double()
    lh = head_lse[:, :rows].double()
    tail_o, tail_l = _tail(go.double(), gl.double(), det.double(), dl.double(),
                           None if old_lse is None else old_lse.double(),
                           None if center is None else center.double())
    c = torch.maximum(lh, tail_l)
    wh = torch.exp(lh - c)
    wt = torch.exp(tail_l - c)
    den = torch.clamp(wh + wt, min=1e-30)
    out[:, :rows] = ((oh * wh[..., None] + tail_o * wt[..., None]) / den[..., None]).float()
    return out


def refresh_detail(full_o, full_lse, head_o, head_lse, go, gl, perm, video_offset, old_det=None,
                   old_dl=None, old_lse=None, center=None):
    """recap/kernels/detail_cache.py:26-186, 304-379.  full_* native order, head_*/go/gl
    reordered.  Returns (det fp16 [banks, rows, d], dl [banks, rows], stats[2] or None)."""
    rows = go.shape[1]
    nat = video_offset + torch.as_tensor(perm[:rows], dtype=torch.long)
    of = full_o[:, nat].double()
    lf = full_lse[:, nat].double()
    oh = head_o[:, :rows].double()
    lh = head_lse[:, :rows].double()
    ratio = torch.clamp(torch.exp(torch.clamp(lh - lf, max=0.0)), max=1.0 - 1e-6)
    den = 1.0 - ratio
    stats = None
    if old_det is not None:
        tail_o, tail_l = _tail(go.double(), gl.double(), old_det.double(), old_dl.double(),
                               None if old_lse is None else old_lse.double(),
                               None if center is None else center.double())
        c = torch.maximum(lh, tail_l)
        wh = torch.exp(lh - c)
        wt = torch.exp(tail_l - c)
        md = torch.clamp(wh + wt, min=1e-30)
        old = (oh * wh[..., None] + tail_o * wt[..., None]) / md[..., None]
        stats = torch.tensor([float(((old - of) ** 2).sum()), float((of ** 2).sum())])
    tail = (of - ratio[..., None] * oh) / den[..., None]
    det = torch.clamp(tail - go.double(), -6e4, 6e4)
    det = torch.where((ratio > 1 - 1e-3)[..., None], torch.zeros_like(det), det)
    dl = torch.clamp(lf + torch.log(den) - gl.double(), -30.0, 30.0)
    return det.to(torch.float16), dl.float(), stats


# ----------------------------------------------------------------------------- the operator


@dataclass
class OracleLayer:
    """Per-layer state of the reference operator (recap/operator.py:33-59 and the basis
    cache of recap/sparse/attention.py:60-70)."""

    basis: torch.Tensor | None = None
    partition: torch.Tensor | None = None  # [banks, nB, nB]
    value: torch.Tensor | None = None
    log_mass: torch.Tensor | None = None
    coarse_lse: torch.Tensor | None = None
    valid: bool = False
    refreshed_at: int = 0
    pending_stats: torch.Tensor | None = None
    pending_age: int | None = None
    trace: dict = field(default_factory=dict)


@dataclass
class OracleOperator:
    """recap/operator.py:153-547 for one stream, single bank group, on CPU.

    ``dtype`` is the model dtype the reference would see (inputs are rounded to it)."""

    permutation: np.ndarray
    text_tokens: int
    text_first: bool
    head_density: float = 0.1
    closure_gate_theta: float = 2.0
    closure_rank: int = 4
    rerank_min_overlap: float = 0.95
    dtype: torch.dtype = torch.bfloat16
    layers: dict = field(default_factory=dict)
    step: int = 0
    basis_override: torch.Tensor | None = None

    def layer(self, i: int) -> OracleLayer:
        return self.layers.setdefault(i, OracleLayer())

    @property
    def n_video(self) -> int:
        return len(self.permutation)

    def _reorder(self, x: torch.Tensor):
        fwd, _ = gather_indices(torch.as_tensor(self.permutation), self.text_tokens, self.text_first)
        return x[..., fwd, :]

    def _restore(self, x: torch.Tensor):
        _, inv = gather_indices(torch.as_tensor(self.permutation), self.text_tokens, self.text_first)
        return x[..., inv, :]

    def _context(self, st: OracleLayer, q_r, k_r, v_r, scale):
        """recap/sparse/attention.py:156-202."""
        nv = self.n_video
        km, counts = pool_blocks(k_r, nv)
        vm, _ = pool_blocks(v_r, nv)
        first = st.basis is None
        if first:
            basis = self.basis_override if self.basis_override is not None else \
                closure_basis(within_block_scatter(k_r, km, counts, nv))
        else:
            basis = st.basis
        var = rotated_variance(k_r, basis, nv)
        cvk = cross_covariance(k_r, v_r, km, counts, nv)
        if first and self.basis_override is None:
            basis, var = order_basis(basis, var, counts)
        st.basis = basis
        var = fold_rank(var, self.closure_rank)
        qsq = rotated_query_square(q_r[:, :nv], basis, self.dtype)
        drift = value_drift(q_r[:, :nv], cvk, scale, self.dtype)
        return dict(km=km, vm=vm, counts=counts, var=var, cvk=cvk, qsq=qsq, drift=drift, basis=basis)

    def _coarse(self, q_r, ctx, partition, scale, rows):
        return coarse_tail(q_r, ctx["km"], ctx["vm"], ctx["var"], ctx["counts"], partition, ctx["qsq"],
                           ctx["drift"], scale, self.closure_gate_theta, rows, self.dtype)

    def _head(self, q_r, k_r, v_r, partition, scale):
        S = q_r.shape[1]
        o, l = masked_attention(q_r, k_r, v_r, kernel_block_mask(partition, S, self.n_video), scale)
        return _rd(o, self.dtype), l

    def refresh(self, i: int, q, k, v):
        """recap/operator.py:253-258, 331-473 for inputs [banks, S, d] in native order."""
        q, k, v = (_rd(t, self.dtype) for t in (q, k, v))
        st = self.layer(i)
        d = q.shape[-1]
        scale = 1.0 / math.sqrt(d)
        nv = self.n_video
        rows = (nv // BLOCK) * BLOCK
        full_o, full_lse = masked_attention(q, k, v, None, scale)
        full_o = _rd(full_o, self.dtype)
        q_r, k_r, v_r = self._reorder(q), self._reorder(k), self._reorder(v)
        revalidating = st.valid
        if not revalidating:
            st.partition = head_partition(q_r, k_r, scale, self.head_density, nv)
        head_o, head_lse = self._head(q_r, k_r, v_r, st.partition, scale)
        ctx = self._context(st, q_r, k_r, v_r, scale)
        go, gl = self._coarse(q_r, ctx, st.partition, scale, rows)
        old_lse = st.coarse_lse if revalidating else None
        center = drift_center(gl, old_lse) if old_lse is not None else None
        det, dl, stats = refresh_detail(
            full_o, full_lse, head_o, head_lse, go, gl, self.permutation, self.text_tokens if self.text_first else 0,
            st.value if revalidating else None, st.log_mass if revalidating else None, old_lse, center)
        st.value, st.log_mass = det, dl
        st.trace = dict(full_o=full_o, full_lse=full_lse, head_o=head_o, head_lse=head_lse, go=go, gl=gl,
                        center=center, ctx=ctx)
        if stats is not None:
            st.pending_stats = stats
            st.pending_age = self.step - st.refreshed_at
        if revalidating:
            new = head_partition(q_r, k_r, scale, self.head_density, nv)
            kept = int((new & st.partition).sum())
            total = max(int(new.sum()), 1)
            st.trace["overlap"] = (kept, total)
            if kept / total >= self.rerank_min_overlap:
                st.coarse_lse = gl.clone()
                st.refreshed_at = self.step
                st.valid = True
                return full_o
            st.partition = new
            head_o, head_lse = self._head(q_r, k_r, v_r, st.partition, scale)
            go, gl = self._coarse(q_r, ctx, st.partition, scale, rows)
            det, dl, _ = refresh_detail(full_o, full_lse, head_o, head_lse, go, gl, self.permutation,
                                        self.text_tokens if self.text_first else 0)
            st.value, st.log_mass = det, dl
        st.coarse_lse = gl.clone()
        st.refreshed_at = self.step
        st.valid = True
        return full_o

    def sparse(self, i: int, q, k, v):
        """recap/operator.py:478-527."""
        q, k, v = (_rd(t, self.dtype) for t in (q, k, v))
        st = self.layer(i)
        if not st.valid:
            raise RuntimeError("a sparse call was requested before an exact refresh")
        d = q.shape[-1]
        scale = 1.0 / math.sqrt(d)
        nv = self.n_video
        rows = (nv // BLOCK) * BLOCK
        q_r, k_r, v_r = self._reorder(q), self._reorder(k), self._reorder(v)
        head_o, head_lse = self._head(q_r, k_r, v_r, st.partition, scale)
        ctx = self._context(st, q_r, k_r, v_r, scale)
        go, gl = self._coarse(q_r, ctx, st.partition, scale, rows)
        center = drift_center(gl, st.coarse_lse)
        merged = sparse_merge(head_o, head_lse, go, gl, st.value.float(), st.log_mass, rows, st.coarse_lse,
                              center)
        st.trace = dict(head_o=head_o, head_lse=head_lse, go=go, gl=gl, center=center, ctx=ctx)
        return _rd(self._restore(merged), self.dtype)

    def drain_validation(self):
        """recap/operator.py:531-547."""
        stats, ages = [], []
        for st in self.layers.values():
            if st.pending_stats is not None and st.pending_age is not None:
                stats.append(st.pending_stats)
                ages.append(int(st.pending_age))
            st.pending_stats = None
            st.pending_age = None
        if not stats:
            return None
        num, den = (float(x) for x in torch.stack(stats).sum(0))
        return min(ages), (math.sqrt(num / den) if den > 0 else float("inf"))


# ----------------------------------------------------------------------------- inputs


def config1_inputs(seed: int = 0):
    """Config 1 of the benchmark: 1x2x2048x64 fp32 N(0,1) Q, K, V drawn in order from one
    generator (grid (8,16,16), no text)."""
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(1, 2, 2048, 64, generator=g) for _ in range(3))


def smooth_lowrank(grid, heads: int, dim: int, text_tokens: int, text_first: bool, seed: int,
                   rank: int = 16, noise: float = 0.5, head_slice: slice | None = None,
                   dtype=torch.bfloat16):
    """Seeded synthetic Q/K/V with per-frame spatially smooth low-rank structure:
    X[t,y,x] = sum_r f_r(t,y,x) u_r + noise * eps, f_r a sum of 4 low-frequency cosines with
    a per-frame phase drift; text tokens i.i.d. N(0,1).  Generated per head from
    (seed, tensor, head) so any head slice reproduces the same values.  Returns q, k, v
    [1, heads_in_slice, S, dim] in native order ([text | video] if text_first)."""
    T, H, W = (int(g) for g in grid)
    nv = T * H * W
    hs = range(heads)[head_slice] if head_slice is not None else range(heads)
    tt = torch.arange(T, dtype=torch.float32).view(T, 1, 1)
    yy = torch.arange(H, dtype=torch.float32).view(1, H, 1) / H
    xx = torch.arange(W, dtype=torch.float32).view(1, 1, W) / W
    outs = []
    for tensor in range(3):
        per_head = []
        for h in hs:
            g = torch.Generator().manual_seed(seed * 1_000_003 + tensor * 10_007 + h)
            u = torch.randn(rank, dim, generator=g) / math.sqrt(rank)
            amp = torch.randn(rank, 4, generator=g)
            ky = torch.randint(-2, 3, (rank, 4), generator=g).float()
            kx = torch.randint(-2, 3, (rank, 4), generator=g).float()
            ph = torch.rand(rank, 4, generator=g) * 2 * math.pi
            dr = (torch.rand(rank, 4, generator=g) - 0.5) * 0.6
            f = torch.zeros(rank, T, H, W)
            for c in range(4):
                arg = 2 * math.pi * (ky[:, c].view(rank, 1, 1, 1) * yy + kx[:, c].view(rank, 1, 1, 1) * xx) \
                    + ph[:, c].view(rank, 1, 1, 1) + dr[:, c].view(rank, 1, 1, 1) * tt
                f += amp[:, c].view(rank, 1, 1, 1) * torch.cos(arg)
            x = f.reshape(rank, nv).T @ u + noise * torch.randn(nv, dim, generator=g)
            text = torch.randn(text_tokens, dim, generator=g)
            x = torch.cat([text, x]) if text_first else torch.cat([x, text])
            per_head.append(x)
        outs.append(torch.stack(per_head).unsqueeze(0).to(dtype))
    return tuple(outs)


def perturb3(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seed: int, eps: float = 0.05):
    """(X + eps * N(0,1)) for X = Q, K, V in order, one generator seeded with ``seed``."""
    g = torch.Generator().manual_seed(seed)
    return tuple((x.float() + eps * torch.randn(x.shape, generator=g)).to(x.dtype) for x in (q, k, v))


def perturb_heads(x: torch.Tensor, seed: int, tensor: int, eps: float = 0.05, head_offset: int = 0):
    """x + eps * N(0,1) with one generator per (seed, tensor, head), so that a head slice
    (head_offset = first head of the slice) reproduces the full tensor's values."""
    out = torch.empty_like(x)
    for h in range(x.shape[1]):
        g = torch.Generator().manual_seed(seed * 1_000_003 + tensor * 10_007 + head_offset + h + 77)
        out[:, h] = (x[:, h].float() + eps * torch.randn(x[:, h].shape, generator=g)).to(x.dtype)
    return out
