"""Sparse attention for one layer: block selection and the corrected coarse tail.

Mirrors ``recap/sparse/attention.py`` (``SparseGeometry``, ``SparseAttention`` with
``head_partition``, ``coarse_tail_context`` and ``coarse_tail_apply``), with every step
on the sm_100a kernels of ``librecap_b200.so``:

``prepare``              one gather+pooling pass over the native Q/K/V (reorder, V
                         transposed, block means) - the inputs of everything below;
``head_partition``       top-k key blocks per query block (refresh only);
``coarse_tail_context``  closure statistics: the shared covariance basis (first call of a
                         sample: scatter + ``eigh`` + ordering), the per-block variances in
                         it (rank-folded) and the value-key covariance;
``coarse_tail_apply``    corrected coarse attention over the omitted blocks, with qsq and
                         drift fused, plus the drift centre when a reference LSE is given.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import _lib
from ..config import keep_blocks
from .layout import Layout, gather_rows, sequence_tokens

BLOCK = 128


@dataclass
class SparseGeometry:
    """Model-level data shared by all layers (recap/sparse/attention.py:33-57)."""

    layout: Layout
    block_size: int
    n_blocks: int
    block_counts: torch.Tensor  # [n_blocks] fp32, tokens per video block

    @classmethod
    def build(cls, layout: Layout, block_size: int) -> "SparseGeometry":
        if int(block_size) != BLOCK:
            raise ValueError("the exact block-sparse kernel requires block_size=128")
        n_blocks = math.ceil(layout.video_tokens / block_size)
        counts = torch.full((n_blocks,), float(block_size), dtype=torch.float32)
        counts[-1] = layout.video_tokens - block_size * (n_blocks - 1)
        return cls(layout=layout, block_size=int(block_size), n_blocks=int(n_blocks), block_counts=counts)

    def to(self, device: torch.device) -> None:
        """Move the block counts to ``device``."""
        if self.block_counts.device != device:
            self.block_counts = self.block_counts.to(device)

    def counts_log(self, device: torch.device) -> torch.Tensor:
        return counts_log(self, device)


def counts_log(geometry, device: torch.device) -> torch.Tensor:
    """ln(tokens per video block) on ``device``; works on the reference's SparseGeometry too."""
    cache = geometry.__dict__.setdefault("_recap_b200_counts_log", {})
    key = str(device)
    if key not in cache:
        cache[key] = torch.log(torch.as_tensor(geometry.block_counts).detach().float().cpu()).to(device)
    return cache[key]


@dataclass
class Shapes:
    """Geometry of one layer call (C ABI conventions, include/recap_b200.h)."""

    batch: int
    heads: int
    banks: int
    S: int
    D: int
    n_video: int
    NB: int
    S_pad: int
    nB: int
    nB_pad: int
    rows: int
    dense_start: int

    @classmethod
    def of(cls, query: torch.Tensor, n_video: int) -> "Shapes":
        b, h, s, d = query.shape
        NB = (s + BLOCK - 1) // BLOCK
        nB = (n_video + BLOCK - 1) // BLOCK
        shared = (n_video % BLOCK) != 0 and s > n_video
        return cls(
            batch=b, heads=h, banks=b * h, S=s, D=d, n_video=n_video, NB=NB, S_pad=NB * BLOCK,
            nB=nB, nB_pad=((nB + BLOCK - 1) // BLOCK) * BLOCK, rows=(n_video // BLOCK) * BLOCK,
            dense_start=nB - 1 if shared else nB,
        )


@dataclass
class LayerInputs:
    """Reordered operands of one layer call, produced by one layout-gather launch."""

    shapes: Shapes
    q: torch.Tensor            # [banks, S_pad, D] bf16
    k: torch.Tensor            # [banks, S_pad, D] bf16
    v_t: torch.Tensor          # [banks, D, S_pad] bf16
    q_mean: torch.Tensor | None
    k_mean: torch.Tensor | None   # [banks, nB, D] fp32
    v_mean: torch.Tensor | None
    k_mean_bf16: torch.Tensor | None  # [banks, nB_pad, D]
    v_mean_t_bf16: torch.Tensor | None  # [banks, D, nB_pad]
    k_centred_t: torch.Tensor | None = None  # [banks, D, S_pad] bf16, block-centred video keys
    variance: torch.Tensor | None = None  # [banks, nB, D] fp32 rank-folded (when the basis was known)
    variance_bf16: torch.Tensor | None = None  # [banks, nB_pad, D]
    k_norm_max: torch.Tensor | None = None  # [banks, NB] fp32 largest |k| per 128-token block
    k_mean_norm: torch.Tensor | None = None  # [banks, nB] fp32 |bf16(kbar)| per video block


class Launches:
    """Counts kernel launches and, when enabled, times each C-ABI call with CUDA events on
    the launching stream."""

    def __init__(self) -> None:
        self.count = 0
        self.timing = False
        self.events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def run(self, name: str, n_kernels: int, *args) -> None:
        if self.timing:
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            _lib.call(name, *args)
            end.record()
            self.events.append((name, start, end))
        else:
            _lib.call(name, *args)
        self.count += n_kernels

    def take_times(self) -> dict[str, list[float]]:
        """Milliseconds per call name since the last take (synchronises)."""
        out: dict[str, list[float]] = {}
        if self.events:
            self.events[-1][2].synchronize()
        for name, a, b in self.events:
            out.setdefault(name, []).append(a.elapsed_time(b))
        self.events = []
        return out


class SparseAttention:
    """Per-layer state: the shared covariance basis, computed once per sample."""

    def __init__(self, geometry: SparseGeometry, config, launches: Launches | None = None):
        self.geometry = geometry
        self.config = config
        self.launches = launches if launches is not None else Launches()
        self._basis: torch.Tensor | None = None      # [banks, D, D] fp32, ordered columns
        self._basis_t: torch.Tensor | None = None    # [banks, D, D] bf16, transposed

    def reset(self) -> None:
        """Forget the basis."""
        self._basis = None
        self._basis_t = None

    @property
    def basis(self) -> torch.Tensor | None:
        return self._basis

    # -- the one pass over the native inputs ----------------------------------------------

    @torch.no_grad()
    def prepare(
        self,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        *,
        q_mean: bool,
        means: bool = True,
        shards=None,
    ) -> LayerInputs:
        """One layout pass.  ``shards`` (a ``recap_b200.ulysses.ShardedIO``): Q, K and V are the
        token shards of the ranks of a sequence-parallel layer, read in place over NVLink;
        ``query``, ``key`` and ``value`` are then unused."""
        layout = self.geometry.layout
        if shards is not None:
            query = shards.shape_carrier()
        if query.shape[-2] != sequence_tokens(layout):
            raise ValueError(
                f"sequence {query.shape[-2]} != video+text {sequence_tokens(layout)}"
            )
        sh = Shapes.of(query, layout.video_tokens)
        dev = query.device if shards is None else shards.device
        bf = torch.bfloat16
        q_r = torch.empty(sh.banks, sh.S_pad, sh.D, dtype=bf, device=dev)
        k_r = torch.empty_like(q_r)
        v_t = torch.empty(sh.banks, sh.D, sh.S_pad, dtype=bf, device=dev)
        qm = km = vm = kmb = vmtb = kct = var = var_bf16 = kmn = None
        basis = None
        knm = torch.empty(sh.banks, sh.S_pad // 128, dtype=torch.float32, device=dev)
        rank = int(self.config.closure_rank)
        if means:
            f32 = torch.float32
            km = torch.empty(sh.banks, sh.nB, sh.D, dtype=f32, device=dev)
            vm = torch.empty_like(km)
            qm = torch.empty_like(km) if q_mean else None
            kmb = torch.zeros(sh.banks, sh.nB_pad, sh.D, dtype=bf, device=dev)
            vmtb = torch.zeros(sh.banks, sh.D, sh.nB_pad, dtype=bf, device=dev)
            kct = torch.empty(sh.banks, sh.D, sh.S_pad, dtype=bf, device=dev)
            kmn = torch.empty(sh.banks, sh.nB, dtype=f32, device=dev)
            if (self._basis is not None and 0 < rank < sh.D and rank <= _lib.load().recap_gather_max_rank()
                    and self._basis.shape == (sh.banks, sh.D, sh.D)):
                basis = self._basis
                var = torch.empty(sh.banks, sh.nB, sh.D, dtype=f32, device=dev)
                var_bf16 = torch.zeros(sh.banks, sh.nB_pad, sh.D, dtype=bf, device=dev)
        if shards is not None:
            entry = shards.gather_call()
        else:
            strides = _strides3(query, key, value)
            entry = ("recap_layout_gather", _lib.ptr(query), _lib.ptr(key), _lib.ptr(value), strides, sh.batch,
                     sh.heads)
        self.launches.run(
            entry[0], 1, *entry[1:],
            sh.S, sh.D, sh.n_video, _lib.ptr(gather_rows(layout, dev)),
            _lib.ptr(q_r), _lib.ptr(k_r), _lib.ptr(v_t), _lib.ptr(qm), _lib.ptr(km), _lib.ptr(vm),
            _lib.ptr(kmb), _lib.ptr(vmtb), _lib.ptr(kct), _lib.ptr(basis), rank if basis is not None else 0,
            _lib.ptr(var), _lib.ptr(var_bf16), _lib.ptr(knm), _lib.ptr(kmn), _lib.stream_handle(dev),
        )
        return LayerInputs(sh, q_r, k_r, v_t, qm, km, vm, kmb, vmtb, kct, var, var_bf16, knm, kmn)

    # -- the partition --------------------------------------------------------------------

    @torch.no_grad()
    def head_partition(self, inputs: LayerInputs, scale: float) -> torch.Tensor:
        """Boolean ``[batch, heads, query blocks, key blocks]`` mask of the selected blocks."""
        sh = inputs.shapes
        if inputs.q_mean is None or inputs.k_mean is None:
            raise ValueError("head_partition needs the query and key block means")
        keep = keep_blocks(self.config.head_density, sh.nB)
        part = torch.empty(sh.batch, sh.heads, sh.nB, sh.nB, dtype=torch.bool, device=inputs.q.device)
        self.launches.run(
            "recap_pool_select", 1,
            _lib.ptr(inputs.q_mean), _lib.ptr(inputs.k_mean), sh.banks, sh.nB, sh.D, keep,
            float(scale), sh.n_video, BLOCK, _lib.ptr(part), _lib.stream_handle(part.device),
        )
        return part

    # -- the moment statistics ------------------------------------------------------------

    @torch.no_grad()
    def coarse_tail_context(self, inputs: LayerInputs, scale: float) -> dict:
        """Closure statistics that do not depend on the partition
        (recap/sparse/attention.py:98-202): C_vk on tensor cores every call; the basis at
        the first call of a sample (scatter, eigh, ordering by pooled variance); the
        rank-folded per-block variances (from the layout pass when the basis was known)."""
        sh = inputs.shapes
        dev = inputs.q.device
        f32 = torch.float32
        rank = int(self.config.closure_rank)
        stream = _lib.stream_handle(dev)
        lib = _lib.load()
        if inputs.k_centred_t is None:
            raise ValueError("coarse_tail_context needs the layout pass's block means and centred keys")
        ws = torch.empty(int(lib.recap_cvk_workspace_floats(sh.banks, sh.D, sh.n_video)), dtype=f32, device=dev)
        cvk = torch.empty(sh.banks, sh.D, sh.D, dtype=f32, device=dev)
        cvk_bf16 = torch.empty(sh.banks, sh.D, sh.D, dtype=torch.bfloat16, device=dev)
        self.launches.run(
            "recap_value_key_covariance", 2, _lib.ptr(inputs.v_t), _lib.ptr(inputs.k_centred_t), sh.banks, sh.S,
            sh.D, sh.n_video, _lib.ptr(ws), _lib.ptr(cvk), _lib.ptr(cvk_bf16), None, stream,
        )
        variance, variance_bf16 = inputs.variance, inputs.variance_bf16

        def full_variance(basis, fold):
            """Per-block variances of every basis column (the first call's ordering needs
            them all), folded to `fold` (0: not folded)."""
            out = torch.empty(sh.banks, sh.nB, sh.D, dtype=f32, device=dev)
            out_bf16 = torch.zeros(sh.banks, sh.nB_pad, sh.D, dtype=torch.bfloat16, device=dev)
            self.launches.run(
                "recap_closure_stats", 1,
                _lib.ptr(inputs.k), _lib.ptr(inputs.v_t), _lib.ptr(inputs.k_mean), sh.banks, sh.S, sh.D,
                sh.n_video, fold, _lib.ptr(basis), None, None, None, _lib.ptr(out), _lib.ptr(out_bf16), None,
                stream,
            )
            return out, out_bf16

        if self._basis is None:
            # first call of the sample: scatter -> eigenbasis -> order by pooled variance
            scatter = torch.empty(sh.banks, sh.D, sh.D, dtype=f32, device=dev)
            sws = torch.empty(int(lib.recap_closure_workspace_floats(sh.banks, sh.D, sh.n_video)), dtype=f32,
                              device=dev)
            self.launches.run(
                "recap_closure_stats", 2,
                _lib.ptr(inputs.k), _lib.ptr(inputs.v_t), _lib.ptr(inputs.k_mean), sh.banks, sh.S, sh.D,
                sh.n_video, 0, None, _lib.ptr(scatter), None, None, None, None, _lib.ptr(sws), stream,
            )
            symmetric = 0.5 * (scatter + scatter.transpose(-1, -2))
            _, evecs = torch.linalg.eigh(symmetric)
            evecs = _orthonormalize(evecs)
            unsorted, _ = full_variance(evecs, 0)
            counts = self.geometry.block_counts.to(dev).reshape(1, -1, 1)
            pooled = (unsorted * counts).sum(1) / counts.sum().clamp_min(1.0)
            order = torch.argsort(pooled, dim=-1, descending=True)
            basis = torch.gather(evecs, 2, order.unsqueeze(1).expand(-1, sh.D, -1)).contiguous()
            basis_t = torch.empty(sh.banks, sh.D, sh.D, dtype=torch.bfloat16, device=dev)
            self.launches.run("recap_basis_prep", 1, _lib.ptr(basis), sh.banks, sh.D, _lib.ptr(basis_t), stream)
            self._basis, self._basis_t = basis, basis_t
            variance, variance_bf16 = full_variance(basis, rank)
        else:
            if self._basis.shape[0] != sh.banks or self._basis.shape[-1] != sh.D:
                raise ValueError("cached basis does not match this call's banks/head_dim")
            if variance is None:
                variance, variance_bf16 = full_variance(self._basis, rank)
        return {
            "variance": variance, "variance_bf16": variance_bf16, "cvk": cvk, "cvk_bf16": cvk_bf16,
            "basis": self._basis, "basis_t": self._basis_t,
        }

    # -- the coarse tail ------------------------------------------------------------------

    @torch.no_grad()
    def coarse_tail_apply(
        self,
        inputs: LayerInputs,
        context: dict,
        partition: torch.Tensor,
        scale: float,
        *,
        old_lse: torch.Tensor | None = None,
        status: torch.Tensor | None = None,
        logit_bound: bool = True,
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
        """Corrected coarse attention over the blocks ``partition`` omits, for the cached
        rows; returns (output bf16 [banks, rows, D], lse fp32 [banks, rows], centre or None).
        ``logit_bound`` lets tiles of block means within the |q| |kbar| logit bound keep the
        running maximum and take the single-pass path (logits, gate and exponentials in one
        loop, no maximum exchange between the two threads of a row); with it off every tile
        computes and exchanges its maximum.  The two agree up to fp32 rounding."""
        sh = inputs.shapes
        dev = inputs.q.device
        out = torch.empty(sh.banks, sh.rows, sh.D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(sh.banks, sh.rows, dtype=torch.float32, device=dev)
        center = partial = None
        if old_lse is not None:
            center = torch.empty(sh.banks, dtype=torch.float32, device=dev)
            partial = torch.empty(sh.banks, max(1, sh.rows // BLOCK), dtype=torch.float32, device=dev)
        if sh.rows == 0:
            if center is not None:
                center.fill_(float("nan"))
            return out, lse, center
        self.launches.run(
            "recap_coarse_tail", 1 + (old_lse is not None),
            _lib.ptr(inputs.q), _lib.ptr(context["basis_t"]), _lib.ptr(context["cvk_bf16"]),
            _lib.ptr(inputs.k_mean_bf16), _lib.ptr(context["variance_bf16"]), _lib.ptr(inputs.v_mean_t_bf16),
            _lib.ptr(partition), _lib.ptr(counts_log(self.geometry, dev)),
            _lib.ptr(inputs.k_mean_norm if logit_bound else None),
            _lib.ptr(old_lse),
            sh.banks, sh.S, sh.D, sh.n_video, float(scale), float(self.config.closure_gate_theta),
            int(self.config.closure_rank), _lib.ptr(out), _lib.ptr(lse), _lib.ptr(partial), _lib.ptr(center),
            _lib.ptr(status),
            _lib.stream_handle(dev),
        )
        return out, lse, center


def _orthonormalize(u: torch.Tensor) -> torch.Tensor:
    """The eigenvectors of an fp32 eigh are orthonormal only to ~3e-5.  The layout pass
    takes the folded tail of the per-block variances from the trace identity
    sum_c var(K U[:, c]) = trace(cov K), which holds for an orthonormal U: two Newton-Schulz
    steps in fp64 (U <- U (3 I - U^T U) / 2, quadratic convergence from 3e-5) make U
    orthonormal to fp32 rounding, moving each vector by ~1e-5, well inside the freedom
    eigh leaves it (signs, rotations within near-degenerate eigenspaces)."""
    x = u.double()
    eye3 = 3.0 * torch.eye(x.shape[-1], dtype=x.dtype, device=x.device)
    for _ in range(2):
        x = 0.5 * x @ (eye3 - x.transpose(-1, -2) @ x)
    return x.float().contiguous()


def _strides3(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    import ctypes

    vals = []
    for t in (q, k, v):
        if t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError("query/key/value must be [batch, heads, sequence, dim] with dim contiguous")
        if t.dtype != torch.bfloat16:
            raise ValueError("the layout kernel takes bf16 inputs")
        vals += [t.stride(0), t.stride(1), t.stride(2)]
    return (ctypes.c_int64 * 9)(*vals)
