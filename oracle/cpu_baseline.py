"""Timed CPU baselines of the corrected SPARSE step - test/benchmark infrastructure only.

The reference has no CPU implementation of its operator (its head is a CUDA extension
and its other kernels are Triton), so the CPU path timed here is the oracle restatement
of the reference's algorithm (``oracle/recap_oracle.py``), in fp32 torch on all host
threads.  Two forms:

* ``FullLayer``: one whole SPARSE layer call, every bank and every query block, no
  sampling (about a minute or more at HunyuanVideo-720p); ``bench.py --impl reference``
  times it.
* ``SampledLayer``: a bounded sample scaled to one layer call, for the GPU arm's
  ``cpu_baseline`` (10-30 s of CPU work) and as a check of its own cost model against the
  whole call:
  - per bank, the work over the whole sequence (layout gather, block pooling of K and V,
    per-block key variances in the basis, C_vk) is timed on ``heads`` banks;
  - per query block, the work over its rows (qsq/drift rows, coarse tail, block-sparse head
    over its kept key blocks, merge) is timed on ``video_qblocks`` evenly spaced video query
    blocks and ``dense_qblocks`` of the dense (text / shared-boundary) query blocks;
  - the layer-call estimate is  H * (t_bank + n_video_qb * t_video_qb + n_dense_qb * t_dense_qb).
"""

from __future__ import annotations

import math
import os
import time

import numpy as np
import torch

from . import recap_oracle as orc

BLOCK = 128


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class SampledLayer:
    """The oracle's REFRESH/SPARSE restricted to sampled query blocks of sampled banks."""

    def __init__(self, spec: dict, heads: int = 2, video_qblocks: int = 48, dense_qblocks: int = 2, seed: int = 0):
        from recap_b200.sparse.geometry import hilbert_permutation  # host-side numpy only

        self.spec = spec
        self.perm = hilbert_permutation(spec["grid"])
        self.nv = len(self.perm)
        self.text = spec["text"]
        self.text_first = spec["text_first"]
        self.S = self.nv + self.text
        self.d = spec["dim"]
        self.scale = 1.0 / math.sqrt(self.d)
        self.nB = (self.nv + BLOCK - 1) // BLOCK
        self.NB = (self.S + BLOCK - 1) // BLOCK
        shared = self.nv % BLOCK != 0 and self.S > self.nv
        self.dense_start = self.nB - 1 if shared else self.nB
        self.rows = (self.nv // BLOCK) * BLOCK
        self.keep = orc.keep_blocks(spec["density"], self.nB)
        self.heads = heads
        n_video_qb = self.rows // BLOCK
        self.video_qb = sorted(set(np.linspace(0, n_video_qb - 1, video_qblocks).round().astype(int).tolist()))
        dense_all = list(range(self.dense_start, self.NB))
        self.dense_qb = dense_all[:dense_qblocks]
        self.n_video_qb_total = n_video_qb
        self.n_dense_qb_total = len(dense_all)
        self.fwd, self.inv = orc.gather_indices(torch.as_tensor(self.perm), self.text, self.text_first)
        torch.set_num_threads(host_threads())
        self.q0, self.k0, self.v0 = (t[0].float() for t in orc.smooth_lowrank(
            spec["grid"], spec["heads"], self.d, self.text, self.text_first, seed, head_slice=slice(0, heads)))
        self._state = None

    # -- the per-bank, whole-sequence part ------------------------------------------------

    def _bank_work(self, q, k, v, basis=None):
        q_r, k_r, v_r = q[:, self.fwd], k[:, self.fwd], v[:, self.fwd]
        km, counts = orc.pool_blocks(k_r, self.nv)
        vm, _ = orc.pool_blocks(v_r, self.nv)
        first = basis is None
        if first:
            basis = orc.closure_basis(orc.within_block_scatter(k_r, km, counts, self.nv))
        var = _rotated_variance_f32(k_r, basis, self.nv)
        cvk = _cross_f32(k_r, v_r, km, counts, self.nv)
        if first:
            basis, var = orc.order_basis(basis, var, counts)
        var = orc.fold_rank(var, 4)
        return dict(q_r=q_r, k_r=k_r, v_r=v_r, km=km, vm=vm, counts=counts, var=var, cvk=cvk, basis=basis)

    # -- the per-query-block part ---------------------------------------------------------

    def _qblock_work(self, ctx, partition, qb, bank_state=None):
        q_r, k_r, v_r = ctx["q_r"], ctx["k_r"], ctx["v_r"]
        kmask = orc.kernel_block_mask(partition, self.S, self.nv)
        r0, r1 = qb * BLOCK, min(self.S, (qb + 1) * BLOCK)
        out = []
        for b in range(self.heads):
            cols = torch.cat([torch.arange(j * BLOCK, min(self.S, (j + 1) * BLOCK))
                              for j in torch.nonzero(kmask[b, qb]).flatten().tolist()])
            s = (q_r[b, r0:r1] @ k_r[b, cols].T) * self.scale
            m = s.max(-1, keepdim=True).values
            p = torch.exp(s - m)
            l = p.sum(-1, keepdim=True)
            oh = (p @ v_r[b, cols]) / l
            lh = (m + torch.log(l)).squeeze(-1)
            if r1 <= self.rows:
                qv = q_r[b:b + 1, r0:r1]
                qsq = orc.rotated_query_square(qv, ctx["basis"][b:b + 1], torch.bfloat16)
                drift = orc.value_drift(qv, ctx["cvk"][b:b + 1], self.scale, torch.bfloat16)
                omitted = ~partition[b, qb]
                kb = ctx["km"][b].to(torch.bfloat16).float()
                vb = ctx["vm"][b].to(torch.bfloat16).float()
                wb = ctx["var"][b].to(torch.bfloat16).float()
                sc = (qv[0] @ kb.T) * self.scale + torch.log(ctx["counts"])
                quad = qsq[0] @ wb.T
                gate = quad * self.scale ** 2 <= 4.0
                sc = sc + torch.where(gate, quad * 0.5 * self.scale ** 2, torch.zeros_like(quad))
                sc[:, ~omitted] = -math.inf
                mc = sc.max(-1, keepdim=True).values
                pc = torch.exp(sc - mc)
                lc = pc.sum(-1, keepdim=True)
                go = (pc.to(torch.bfloat16).float() @ vb) / lc + ((pc * gate).sum(-1, keepdim=True) / lc) * drift[0]
                gl = (mc + torch.log(lc)).squeeze(-1)
                if bank_state is not None:
                    det, dl, ogl, center = (t[b, r0:r1] if t.dim() > 1 else t[b] for t in bank_state)
                    out.append(orc.sparse_merge(oh[None], lh[None], go[None], gl[None], det[None].float(), dl[None],
                                                r1 - r0, ogl[None], center.reshape(1)))
                else:
                    out.append((oh, lh, go, gl))
            else:
                out.append((oh, lh))
        return out

    # -- refresh (untimed) and timed sparse steps ------------------------------------------

    def refresh(self):
        """Partition, basis and a refinement for the sampled rows (dense rows exact)."""
        ctx = self._bank_work(self.q0, self.k0, self.v0)
        part = orc.head_partition(ctx["q_r"], ctx["k_r"], self.scale, self.spec["density"], self.nv)
        det = torch.zeros(self.heads, self.rows, self.d, dtype=torch.float16)
        dl = torch.zeros(self.heads, self.rows)
        ogl = torch.zeros(self.heads, self.rows)
        for qb in self.video_qb:
            r0, r1 = qb * BLOCK, (qb + 1) * BLOCK
            for b, (oh, lh, go, gl) in enumerate(self._qblock_work(ctx, part, qb)):
                s = (ctx["q_r"][b, r0:r1] @ ctx["k_r"][b].T) * self.scale
                lf = torch.logsumexp(s, -1)
                of = torch.softmax(s, -1) @ ctx["v_r"][b]
                ratio = torch.clamp(torch.exp(torch.clamp(lh - lf, max=0)), max=1 - 1e-6)
                tail = (of - ratio[:, None] * oh) / (1 - ratio)[:, None]
                det[b, r0:r1] = torch.clamp(tail - go, -6e4, 6e4).half()
                dl[b, r0:r1] = torch.clamp(lf + torch.log(1 - ratio) - gl, -30, 30)
                ogl[b, r0:r1] = gl
        self._state = dict(basis=ctx["basis"], partition=part, det=det, dl=dl, ogl=ogl)
        self.q1, self.k1, self.v1 = orc.perturb3(self.q0, self.k0, self.v0, seed=1)

    def step(self) -> dict:
        """One timed SPARSE step on the sample; returns the component times (s)."""
        if self._state is None:
            self.refresh()
        st = self._state
        t0 = time.perf_counter()
        ctx = self._bank_work(self.q1, self.k1, self.v1, basis=st["basis"])
        t1 = time.perf_counter()
        center = torch.zeros(self.heads)  # per-bank centre; the sample's own rows stand in
        tv = 0.0
        for qb in self.video_qb:
            a = time.perf_counter()
            self._qblock_work(ctx, st["partition"], qb, (st["det"], st["dl"], st["ogl"], center))
            tv += time.perf_counter() - a
        td = 0.0
        for qb in self.dense_qb:
            a = time.perf_counter()
            self._qblock_work(ctx, st["partition"], qb)
            td += time.perf_counter() - a
        return dict(bank=(t1 - t0) / self.heads, video_qb=tv / (len(self.video_qb) * self.heads),
                    dense_qb=(td / (len(self.dense_qb) * self.heads)) if self.dense_qb else 0.0)

    def layer_us(self, parts: dict, heads_total: int) -> float:
        per_bank = parts["bank"] + self.n_video_qb_total * parts["video_qb"] + \
            self.n_dense_qb_total * parts["dense_qb"]
        return heads_total * per_bank * 1e6

    def sample_text(self) -> str:
        return (f"{self.heads} banks x ({len(self.video_qb)} video + {len(self.dense_qb)} dense) query blocks of "
                f"{self.n_video_qb_total}+{self.n_dense_qb_total}, whole-sequence work per bank timed in full; "
                f"scaled to {self.spec['heads']} banks x all query blocks")


def _rotated_variance_f32(k_r, basis, nv):
    banks, _, d = k_r.shape
    nb = (nv + BLOCK - 1) // BLOCK
    full = (nv // BLOCK) * BLOCK
    r = torch.bmm(k_r[:, :full], basis).reshape(banks, full // BLOCK, BLOCK, d)
    var = ((r - r.mean(2, keepdim=True)) ** 2).mean(2)
    if nb * BLOCK != full:
        rt = torch.bmm(k_r[:, full:nv], basis)
        var = torch.cat([var, ((rt - rt.mean(1, keepdim=True)) ** 2).mean(1, keepdim=True)], 1)
    return var.clamp_min(0.0)


def _cross_f32(k_r, v_r, km, counts, nv):
    blk = torch.arange(nv) // BLOCK
    c = k_r[:, :nv] - km[:, blk]
    return torch.bmm(v_r[:, :nv].transpose(1, 2), c) / counts.sum()


class FullLayer:
    """The oracle port's whole SPARSE layer call - every bank, every query block, no
    sampling - in fp32 torch on all host threads: the timed step of ``bench.py --impl
    reference``.

    ``setup()`` (untimed) builds, per bank, the state a SPARSE step reads from the REFRESH
    before it (recap/operator.py:331-473): the partition, the ordered covariance basis and
    the coarse log-mass of every cached row on the refresh inputs.  The refinement of the
    cached rows is left at zero: its values do not change the arithmetic of the step, and
    computing it needs the dense pass over every row (174 TFLOP at config 4, far beyond a
    bounded CPU run).  ``step()`` then runs recap/operator.py:478-527 for every bank: the
    reorder, block pooling, per-block variances in the basis and C_vk, qsq and drift, the
    coarse tail of every cached row, the block-sparse head of every query block over its
    kept key blocks, the drift-weighted merge and the restore."""

    def __init__(self, spec: dict, seed: int = 0, heads: int | None = None):
        from recap_b200.sparse.geometry import hilbert_permutation  # host-side numpy only

        self.spec = spec
        self.perm = hilbert_permutation(spec["grid"])
        self.nv = len(self.perm)
        self.text = spec["text"]
        self.text_first = spec["text_first"]
        self.S = self.nv + self.text
        self.d = spec["dim"]
        self.scale = 1.0 / math.sqrt(self.d)
        self.nB = (self.nv + BLOCK - 1) // BLOCK
        self.NB = (self.S + BLOCK - 1) // BLOCK
        self.rows = (self.nv // BLOCK) * BLOCK
        # banks of the layer call: heads x batch (a batch's banks draw further head indices)
        self.heads = spec["heads"] * spec.get("batch", 1) if heads is None else int(heads)
        self.seed = seed
        self.fwd, self.inv = orc.gather_indices(torch.as_tensor(self.perm), self.text, self.text_first)
        torch.set_num_threads(host_threads())
        self.state: list[dict] = []
        self.inputs: list[tuple] = []

    def _bank_inputs(self, h: int):
        x0 = [t[0, 0] for t in orc.smooth_lowrank(self.spec["grid"], max(self.spec["heads"], h + 1), self.d, self.text,
                                                   self.text_first, self.seed, head_slice=slice(h, h + 1))]
        x1 = [orc.perturb_heads(t[None, None], seed=1, tensor=i, head_offset=h)[0, 0] for i, t in enumerate(x0)]
        return x0, x1

    def setup(self) -> None:
        """Untimed: per bank, the REFRESH state on the first inputs, and the step's inputs."""
        self.state, self.inputs = [], []
        for h in range(self.heads):
            x0, x1 = self._bank_inputs(h)
            q_r, k_r, v_r = (t.float()[self.fwd] for t in x0)
            part = orc.head_partition(q_r[None], k_r[None], self.scale, self.spec["density"], self.nv)[0]
            km, counts = orc.pool_blocks(k_r[None], self.nv)
            b0 = orc.closure_basis(orc.within_block_scatter(k_r[None], km, counts, self.nv))
            basis, _ = orc.order_basis(b0, _rotated_variance_f32(k_r[None], b0, self.nv), counts)
            st = dict(partition=part, basis=basis[0])
            _, gl, _ = self._coarse(q_r, k_r, v_r, st)
            st.update(ogl=gl, det=torch.zeros(self.rows, self.d, dtype=torch.float16), dl=torch.zeros(self.rows))
            self.state.append(st)
            self.inputs.append(tuple(x1))  # model dtype (bf16), native order

    def _coarse(self, q_r, k_r, v_r, st):
        """Closure statistics and the coarse tail of every cached row (fp32, the
        reference's bf16 rounding points)."""
        nv, rows, d, sc = self.nv, self.rows, self.d, self.scale
        bf = torch.bfloat16

        def rd(x):
            return x.to(bf).float()

        km, counts = orc.pool_blocks(k_r[None], nv)
        vm, _ = orc.pool_blocks(v_r[None], nv)
        var = orc.fold_rank(_rotated_variance_f32(k_r[None], st["basis"][None], nv), 4)[0]
        cvk = _cross_f32(k_r[None], v_r[None], km, counts, nv)[0]
        qv = rd(q_r[:rows])
        qsq = rd(rd(qv @ rd(st["basis"])) ** 2)
        drift = rd(sc * rd(qv @ rd(cvk).T))
        kb, vb, wb = rd(km[0]), rd(vm[0]), rd(var)
        logn = torch.log(counts.float())
        go = torch.empty(rows, d)
        gl = torch.empty(rows)
        s2 = sc * sc
        nqb = rows // BLOCK
        for c0 in range(0, nqb, 32):
            c1 = min(nqb, c0 + 32)
            r0, r1 = c0 * BLOCK, c1 * BLOCK
            s = (qv[r0:r1] @ kb.T) * sc + logn
            quad = qsq[r0:r1] @ wb.T
            gate = quad * s2 <= 4.0
            s = s + torch.where(gate, quad * (0.5 * s2), torch.zeros_like(quad))
            s.masked_fill_(st["partition"][c0:c1].repeat_interleave(BLOCK, dim=0), -math.inf)
            m = s.max(-1, keepdim=True).values
            m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
            p = torch.exp(s - m)
            l = p.sum(-1, keepdim=True)
            g = (p * gate).sum(-1, keepdim=True) / l
            o = rd((rd(p) @ vb) / l)
            go[r0:r1] = rd(o + rd(rd(g) * drift[r0:r1]))
            gl[r0:r1] = (m + torch.log(l)).squeeze(-1)
        return go, gl, counts

    def sparse_bank(self, q, k, v, st: dict) -> torch.Tensor:
        """One bank's SPARSE call: native [S, d] model-dtype inputs in, native fp32 out."""
        q_r, k_r, v_r = (t.float()[self.fwd] for t in (q, k, v))
        S, d, sc, rows = self.S, self.d, self.scale, self.rows
        go, gl, _ = self._coarse(q_r, k_r, v_r, st)
        center = (gl - st["ogl"]).mean()
        kmask = orc.kernel_block_mask(st["partition"][None], S, self.nv)[0]
        pad = self.NB * BLOCK - S
        kp = torch.nn.functional.pad(k_r, (0, 0, 0, pad)).view(self.NB, BLOCK, d)
        vp = torch.nn.functional.pad(v_r, (0, 0, 0, pad)).view(self.NB, BLOCK, d)
        oh = torch.empty(S, d)
        lh = torch.empty(S)
        for i in range(self.NB):
            r0, r1 = i * BLOCK, min(S, (i + 1) * BLOCK)
            blocks = torch.nonzero(kmask[i]).flatten()
            s = (q_r[r0:r1] @ kp[blocks].reshape(-1, d).T) * sc
            if pad and bool(blocks[-1] == self.NB - 1):
                s[:, -pad:] = -math.inf  # padding past the end of the sequence
            m = s.max(-1, keepdim=True).values
            p = torch.exp(s - m)
            l = p.sum(-1, keepdim=True)
            oh[r0:r1] = (p @ vp[blocks].reshape(-1, d)) / l
            lh[r0:r1] = (m + torch.log(l)).squeeze(-1)
        oh = oh.to(torch.bfloat16).float()
        out = oh.clone()
        if rows:
            admit = torch.exp(-(gl - st["ogl"] - center).abs())
            cl = gl + st["dl"]
            tc = torch.maximum(gl, cl)
            ms = (1 - admit) * torch.exp(gl - tc)
            mc = admit * torch.exp(cl - tc)
            den = torch.clamp(ms + mc, min=1e-30)
            tail_o = (go * ms[:, None] + (go + st["det"].float()) * mc[:, None]) / den[:, None]
            tail_l = tc + torch.log(den)
            c = torch.maximum(lh[:rows], tail_l)
            wh = torch.exp(lh[:rows] - c)
            wt = torch.exp(tail_l - c)
            out[:rows] = (oh[:rows] * wh[:, None] + tail_o * wt[:, None]) / torch.clamp(wh + wt, min=1e-30)[:, None]
        return out.to(torch.bfloat16).float()[self.inv]

    def step(self) -> float:
        """One whole SPARSE layer call over every bank; returns its wall seconds."""
        t0 = time.perf_counter()
        for x, st in zip(self.inputs, self.state):
            self.sparse_bank(*x, st)
        return time.perf_counter() - t0


def time_sparse_sample(op=None, inputs=None, layout=None, spec=None, repeats: int = 2) -> dict:
    """cpu_baseline entry for bench.py: median of ``repeats`` sampled steps, scaled."""
    runner = SampledLayer(spec)
    runner.refresh()
    runner.step()  # warm-up
    banks = spec["heads"] * spec.get("batch", 1)
    vals = sorted(runner.layer_us(runner.step(), banks) for _ in range(repeats))
    sample = runner.sample_text() + (f"; x{spec['batch']} for the layer's batch" if spec.get("batch", 1) > 1 else "")
    return {"value": round(vals[len(vals) // 2], 1), "unit": "us/layer", "cores": host_threads(),
            "torch_threads": torch.get_num_threads(), "kind": "port", "sample": sample}


def reference_arm(spec: dict, metric: str, unit: str, steps: int, warmup: int, config: dict | None = None) -> dict:
    """``bench.py --impl reference``: the reference's CPU path (the oracle port, fp32 torch on
    all host threads) on the same workload as the GPU arm.

    The timed region is ONE whole, unsampled SPARSE layer call (``FullLayer.step``: every
    bank, every query block), whatever ``steps`` asks: a layer call is a minute or more of
    CPU work, so the run reports ``steps_timed`` = 1.  The ``warmup`` steps run on the
    bounded sample of ``SampledLayer``, whose scaled figure is reported beside the value as
    a check of its cost model (``sampled_estimate_us``)."""
    runner = SampledLayer(spec)
    runner.refresh()
    for _ in range(max(1, warmup)):
        runner.step()
    est = sorted(runner.layer_us(runner.step(), spec["heads"] * spec.get("batch", 1)) for _ in range(2))
    sampled = est[len(est) // 2]
    full = FullLayer(spec)
    t_setup = time.perf_counter()
    full.setup()
    t_setup = time.perf_counter() - t_setup
    wall = full.step()
    value = round(wall * 1e6, 1)
    return {
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "higher_is_better": False,
        "ms_per_step": round(value / 1000.0, 3), "steps_timed": 1, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (the GPU arm's generator restated on the CPU)",
        "config": config if config is not None else {"workload": spec["name"]},
        "cpu_baseline": {
            "value": value, "unit": unit, "kind": "port", "cores": host_threads(),
            "torch_threads": torch.get_num_threads(),
            "sample": f"one whole SPARSE layer call: {full.heads} banks x all {full.NB} query blocks, no sampling "
                      f"(refresh state built untimed in {t_setup:.0f} s)",
            "sampled_estimate_us": round(sampled, 1),
            "sampled_estimate_sample": runner.sample_text(),
        },
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
