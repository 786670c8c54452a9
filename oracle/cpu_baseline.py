"""Timed CPU baseline of the corrected SPARSE step - test/benchmark infrastructure only.

The reference has no CPU implementation of its operator (its head is a CUDA extension
and its other kernels are Triton), so the CPU path timed here is the oracle restatement
of the reference's algorithm (``oracle/recap_oracle.py``), in fp32 torch on all host
threads.  A full HunyuanVideo-720p layer call is minutes of CPU work, so one step times a
bounded sample and scales it to one layer call:

* per bank, the work over the whole sequence (layout gather, block pooling of K and V,
  per-block key variances in the basis, C_vk) is timed on ``heads`` banks;
* per query block, the work over its rows (qsq/drift rows, coarse tail, block-sparse head
  over its kept key blocks, merge) is timed on ``video_qblocks`` evenly spaced video query
  blocks and ``dense_qblocks`` of the dense (text / shared-boundary) query blocks;
* the layer-call estimate is  H * (t_bank + n_video_qb * t_video_qb + n_dense_qb * t_dense_qb).
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


def time_sparse_sample(op=None, inputs=None, layout=None, spec=None, repeats: int = 2) -> dict:
    """cpu_baseline entry for bench.py: median of ``repeats`` sampled steps, scaled."""
    runner = SampledLayer(spec)
    runner.refresh()
    runner.step()  # warm-up
    vals = sorted(runner.layer_us(runner.step(), spec["heads"]) for _ in range(repeats))
    return {"value": round(vals[len(vals) // 2], 1), "unit": "us/layer", "cores": host_threads(),
            "torch_threads": torch.get_num_threads(), "kind": "port", "sample": runner.sample_text()}


def reference_arm(spec: dict, metric: str, unit: str, steps: int, warmup: int) -> dict:
    """``bench.py --impl reference``: the reference's CPU path (the oracle port) on all host
    threads, one sampled SPARSE step per benchmark step, scaled to one layer call."""
    runner = SampledLayer(spec)
    runner.refresh()
    for _ in range(warmup):
        runner.step()
    t0 = time.perf_counter()
    vals = [runner.layer_us(runner.step(), spec["heads"]) for _ in range(steps)]
    wall = time.perf_counter() - t0
    value = round(float(np.mean(vals)), 1)
    return {
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "higher_is_better": False,
        "ms_per_step": round(value / 1000.0, 3), "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (same generator as the GPU arm, CPU)",
        "config": {"workload": spec["name"], "heads": spec["heads"], "head_dim": spec["dim"]},
        "cpu_baseline": {"value": value, "unit": unit, "kind": "port", "cores": host_threads(),
                         "sample": runner.sample_text(), "sample_wall_s_per_step": round(wall / steps, 2)},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
