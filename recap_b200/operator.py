"""Attention for the EXACT, REFRESH and SPARSE steps, on B200.

Drop-in for ``recap.operator`` (recap/operator.py): the same ``Operator.build``,
``reset``, ``banks_valid``, ``begin_step``, ``set_stream``, ``attend``,
``drain_validation`` and ``peak_bank_bytes``, the same ``DetailBank`` fields and the same
re-selection and validation state machine, so ``recap.session.RecapSession``, the
controller and the model processors run on it unchanged.  Every tensor operation of a
call runs in ``librecap_b200.so``:

``EXACT``    one layout pass + the attention kernel over every key block.
``REFRESH``  block selection, then one attention pass that gives the dense output with LSE
             and the block-sparse head on the way, the coarse tail and the refinement write
             (scoring the old refinement first when one exists).
``SPARSE``   one layout pass, the closure statistics, the coarse tail (with the drift
             centre) and the block-sparse attention whose epilogue merges head, coarse tail
             and drift-weighted refinement and writes native order.

Inputs are ``[batch, heads, sequence, dim]`` in the model's native token order (any
strides with ``dim`` contiguous).  The kernels compute in bf16 with fp32 accumulation;
other input dtypes are cast to bf16 on entry and the output is cast back.

Head parallelism: with ``process_group`` set, each rank holds a slice of the heads; the
whole-layer re-selection decision and the validation sums are all-reduced over the group,
so every rank takes the same decision the single-GPU operator would.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, fields

import torch

from . import _lib
from .config import OperatorConfig
from .sparse.attention import Launches, LayerInputs, SparseAttention, SparseGeometry
from .sparse.layout import Layout, gather_rows, video_offset, video_permutation_i32

EXACT = "exact"
REFRESH = "refresh"
SPARSE = "sparse"


def layer_counts_sum(counts: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the (kept, total) overlap counts of this rank's heads over the process group, in
    place and without a host read: the reference takes the re-selection decision over the
    whole layer (recap/operator.py:282-291, 425-428), and with head sharding the layer
    spans ranks."""
    if group is not None:
        import torch.distributed as dist

        dist.all_reduce(counts, group=group)
    return counts


def layer_counts_reduce(counts: torch.Tensor, group=None) -> tuple[int, int]:
    """``layer_counts_sum`` and the host read of the two sums."""
    kept, total = (int(x) for x in layer_counts_sum(counts, group).cpu())
    return kept, total


def keep_partition(kept: int, total: int, min_overlap: float) -> bool:
    """Keep the old partition iff the new selection overlaps it by at least min_overlap
    (recap/operator.py:425-428)."""
    return kept / max(total, 1) >= float(min_overlap)


def validation_reduce(total: torch.Tensor, group=None) -> tuple[float, float]:
    """Sum (sum err^2, sum ref^2) over the process group (recap/operator.py:544-545)."""
    if group is not None:
        import torch.distributed as dist

        dist.all_reduce(total, group=group)
    numerator, denominator = (float(x) for x in total)
    return numerator, denominator


def _bank_fits(bank: "DetailBank", sh) -> bool:
    """Whether a bank's partition and refinement have this call's shapes."""
    return (bank.partition is not None and tuple(bank.partition.shape) == (sh.batch, sh.heads, sh.nB, sh.nB)
            and bank.value is not None and tuple(bank.value.shape) == (sh.banks, sh.rows, sh.D)
            and bank.log_mass is not None and bank.coarse_lse is not None
            and tuple(bank.coarse_lse.shape) == (sh.banks, sh.rows))


@dataclass
class DetailBank:
    """What a layer keeps between a REFRESH and the SPARSE steps after it: the selected
    key blocks and the cached correction of the tail.  The field names and dtypes are those
    of recap/operator.py:33-59, which the host-bank streaming and the session read."""

    # selected key blocks per query block, [batch, heads, nB, nB] bool
    partition: torch.Tensor | None = None
    # the correction stored at the refresh: tail value ([banks, rows, dim] fp16) and tail
    # log-mass ([banks, rows] fp32)
    value: torch.Tensor | None = None
    log_mass: torch.Tensor | None = None
    # the coarse tail's log-mass at that refresh ([banks, rows] fp32): the drift weight of
    # a later step compares the fresh coarse log-mass against it
    coarse_lse: torch.Tensor | None = None
    valid: bool = False
    refreshed_at: int = 0
    # (sum of squared error, sum of squared dense output) of the previous correction,
    # scored at this refresh ([2] fp32), and that correction's age in steps
    pending_stats: torch.Tensor | None = None
    pending_age: int | None = None
    sequence_tokens: int = 0
    n_video: int = 0
    _mask: torch.Tensor | None = field(default=None, repr=False)

    @property
    def head_kernel_mask(self) -> torch.Tensor | None:
        """``[banks, blocks, blocks]`` bool mask on the kernel's 128-token grid (built on
        demand from the partition; the kernels read the partition directly)."""
        if self.partition is None:
            return None
        if self._mask is None:
            b, h, nb, _ = self.partition.shape
            NB = (self.sequence_tokens + 127) // 128
            mask = torch.empty(b * h, NB, NB, dtype=torch.bool, device=self.partition.device)
            _lib.call(
                "recap_kernel_block_mask", _lib.ptr(self.partition), b * h, self.sequence_tokens,
                self.n_video, _lib.ptr(mask), _lib.stream_handle(mask.device),
            )
            self._mask = mask
        return self._mask

    def set_partition(self, partition: torch.Tensor, sequence_tokens: int, n_video: int) -> None:
        self.partition = partition
        self.sequence_tokens = int(sequence_tokens)
        self.n_video = int(n_video)
        self._mask = None

    def release(self) -> None:
        """Back to the state of a bank that was never refreshed."""
        for f in fields(self):
            setattr(self, f.name, f.default)


@dataclass
class Operator:
    """Dispatches one attention call per layer and owns the detail banks."""

    config: OperatorConfig
    layout: Layout
    #: per-layer sparse state, indexed ``[stream][layer]``
    layers: list[list[SparseAttention]]
    banks: list[list[DetailBank]] = field(default_factory=list)
    kind: str = EXACT
    step: int = 0
    stream: int = 0
    refreshed_layers: int = 0
    process_group: object | None = None
    launches: Launches = field(default_factory=Launches)
    _status: dict = field(default_factory=dict, repr=False)

    def __post_init__(self) -> None:
        if not self.layers or isinstance(self.layers[0], SparseAttention):
            raise TypeError("Operator.layers must be indexed [stream][layer]")
        self.banks = [[DetailBank() for _ in row] for row in self.layers]
        for row in self.layers:
            for layer in row:
                layer.launches = self.launches

    @classmethod
    def build(
        cls,
        config: OperatorConfig,
        geometry: SparseGeometry,
        *,
        n_layers: int,
        n_streams: int = 1,
        process_group=None,
    ) -> "Operator":
        """An operator with a ``SparseAttention`` state (basis of the sample) and a bank for
        every layer of every guidance stream."""
        if min(n_layers, n_streams) < 1:
            raise ValueError("n_layers and n_streams must be positive")
        if int(getattr(config, "block_size", 128)) != 128:
            raise ValueError("the exact block-sparse kernel requires block_size=128")
        per_stream = lambda: [SparseAttention(geometry, config) for _ in range(n_layers)]  # noqa: E731
        return cls(config, geometry.layout, [per_stream() for _ in range(n_streams)], process_group=process_group)

    @property
    def n_streams(self) -> int:
        return len(self.layers)

    def _all_banks(self):
        return (bank for row in self.banks for bank in row)

    def reset(self) -> None:
        """A new sample: every bank empty, every basis forgotten, the step counters at zero."""
        for bank in self._all_banks():
            bank.release()
        for layer in (layer for row in self.layers for layer in row):
            layer.reset()
        self.kind, self.step, self.stream, self.refreshed_layers = EXACT, 0, 0, 0

    @property
    def banks_valid(self) -> bool:
        """True once every layer of every stream has stored a correction."""
        banks = list(self._all_banks())
        return bool(banks) and all(bank.valid for bank in banks)

    def begin_step(self, step: int, kind: str) -> None:
        """Start a denoising step of the given kind; the calls that follow use it."""
        if kind not in (EXACT, REFRESH, SPARSE):
            raise ValueError(f"unknown computed call kind {kind!r}")
        self.step, self.kind, self.stream, self.refreshed_layers = int(step), kind, 0, 0

    def set_stream(self, stream: int) -> None:
        """Select the guidance stream whose banks the next calls use."""
        if stream < 0 or stream >= self.n_streams:
            raise ValueError(f"stream {stream} outside 0..{self.n_streams - 1}")
        self.stream = int(stream)

    # -- device status ---------------------------------------------------------------------

    def status_word(self, device: torch.device) -> torch.Tensor:
        key = str(device)
        word = self._status.get(key)
        if word is None:
            word = torch.zeros(1, dtype=torch.int32, device=device)
            self._status[key] = word
        return word

    def check_device_status(self) -> None:
        """Raise if a kernel gave up waiting on an on-chip barrier (synchronises)."""
        for word in self._status.values():
            code = int(word.item())
            if code:
                word.zero_()
                raise RuntimeError(
                    f"a recap_b200 kernel reported a device timeout: "
                    f"{_lib.STATUS_NAMES.get(code, code)}"
                )

    # -- dispatch --------------------------------------------------------------------------

    @torch.no_grad()
    def attend(
        self,
        layer_index: int,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
    ) -> torch.Tensor:
        """One attention call: ``[b, h, S, d]`` native order in, same shape/dtype out."""
        if not (query.is_cuda and key.is_cuda and value.is_cuda):
            raise ValueError("recap_b200.Operator runs on CUDA tensors only")
        if query.shape != key.shape or key.shape != value.shape:
            raise ValueError("Q/K/V shapes differ")
        in_dtype = query.dtype
        if in_dtype != torch.bfloat16:
            query, key, value = (t.to(torch.bfloat16) for t in (query, key, value))
        layer = self.layers[self.stream][layer_index]
        bank = self.banks[self.stream][layer_index]
        if self.kind == SPARSE:
            out = self._sparse(layer, bank, query, key, value)
        elif self.kind == EXACT:
            out = self._exact(layer, query, key, value)
        else:
            out = self._refresh(layer, bank, query, key, value)
        return out if in_dtype == torch.bfloat16 else out.to(in_dtype)

    @torch.no_grad()
    def attend_sharded(self, layer_index: int, io) -> None:
        """One REFRESH or SPARSE call of a sequence-parallel layer whose Q/K/V projections and
        attention output stay sharded by token over the ranks (``recap_b200.ulysses.ShardedIO``):
        the layout pass reads this rank's heads from every rank's projection buffer, and the
        output rows go to the ranks that own the tokens.  The same arithmetic as ``attend``
        on the gathered heads; the caller orders the ranks' buffer writes around it (a
        collective before and after)."""
        if self.kind not in (REFRESH, SPARSE):
            raise ValueError("sharded attention runs REFRESH and SPARSE calls")
        layer = self.layers[self.stream][layer_index]
        bank = self.banks[self.stream][layer_index]
        if self.kind == SPARSE:
            self._sparse(layer, bank, None, None, None, io=io)
        else:
            out = self._refresh(layer, bank, None, None, None, io=io)
            io.scatter_output(out)

    def _scale(self, query: torch.Tensor) -> float:
        return 1.0 / math.sqrt(query.shape[-1])

    def _dense(self, inputs: LayerInputs, scale: float, status, native: bool = True):
        """Attention over every key block: output and LSE in native order."""
        sh = inputs.shapes
        dev = inputs.q.device
        out = torch.empty(sh.batch, sh.heads, sh.S, sh.D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(sh.banks, sh.S, dtype=torch.float32, device=dev)
        self.launches.run(
            "recap_block_sparse_fmha", 1,
            _lib.ptr(inputs.q), _lib.ptr(inputs.k), _lib.ptr(inputs.v_t), None, _lib.ptr(inputs.k_norm_max),
            sh.banks, sh.S, sh.D,
            sh.n_video, 1, float(scale), _lib.ptr(gather_rows(self.layout, dev)) if native else None,
            _lib.ptr(out), _lib.ptr(lse), _lib.ptr(status), _lib.stream_handle(dev),
        )
        return out, lse

    def _dense_and_head(self, inputs: LayerInputs, partition: torch.Tensor, scale: float, status):
        """One pass over every key block: the dense output and LSE in native order, and the
        block-sparse head output and LSE (kept blocks only) in reordered order."""
        sh = inputs.shapes
        dev = inputs.q.device
        out = torch.empty(sh.batch, sh.heads, sh.S, sh.D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(sh.banks, sh.S, dtype=torch.float32, device=dev)
        head_o = torch.empty(sh.banks, sh.S, sh.D, dtype=torch.bfloat16, device=dev)
        head_lse = torch.empty(sh.banks, sh.S, dtype=torch.float32, device=dev)
        self.launches.run(
            "recap_refresh_attention", 1,
            _lib.ptr(inputs.q), _lib.ptr(inputs.k), _lib.ptr(inputs.v_t), _lib.ptr(partition),
            _lib.ptr(inputs.k_norm_max), sh.banks, sh.S, sh.D, sh.n_video, float(scale),
            _lib.ptr(gather_rows(self.layout, dev)), _lib.ptr(out), _lib.ptr(lse), _lib.ptr(head_o),
            _lib.ptr(head_lse), _lib.ptr(status), _lib.stream_handle(dev),
        )
        return out, lse, head_o, head_lse

    def _head(self, inputs: LayerInputs, partition: torch.Tensor, scale: float, status):
        """Block-sparse head: output and LSE in reordered order."""
        sh = inputs.shapes
        dev = inputs.q.device
        out = torch.empty(sh.banks, sh.S, sh.D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(sh.banks, sh.S, dtype=torch.float32, device=dev)
        self.launches.run(
            "recap_block_sparse_fmha", 1,
            _lib.ptr(inputs.q), _lib.ptr(inputs.k), _lib.ptr(inputs.v_t), _lib.ptr(partition),
            _lib.ptr(inputs.k_norm_max), sh.banks,
            sh.S, sh.D, sh.n_video, 0, float(scale), None, _lib.ptr(out), _lib.ptr(lse), _lib.ptr(status),
            _lib.stream_handle(dev),
        )
        return out, lse

    @torch.no_grad()
    def _exact(self, layer: SparseAttention, query, key, value) -> torch.Tensor:
        inputs = layer.prepare(query, key, value, q_mean=False, means=False)
        out, _ = self._dense(inputs, self._scale(query), self.status_word(query.device))
        return out

    # -- refresh ---------------------------------------------------------------------------

    def _layer_overlap(self, new: torch.Tensor, old: torch.Tensor) -> torch.Tensor:
        """Device int64 (kept, total) = (|new & old|, |new|) over the whole layer (all ranks),
        queued on the stream; the caller reads it on the host when it needs the decision."""
        counts = torch.empty(2, dtype=torch.int64, device=new.device)
        self.launches.run(
            "recap_partition_overlap", 1, _lib.ptr(new), _lib.ptr(old), new.numel(), _lib.ptr(counts),
            _lib.stream_handle(new.device),
        )
        return layer_counts_sum(counts, self.process_group)

    @torch.no_grad()
    def _refresh(self, layer: SparseAttention, bank: DetailBank, query, key, value, io=None) -> torch.Tensor:
        """Dense output; stores the refinement and measures the previous one
        (recap/operator.py:331-473).

        The re-selection test of a revalidating refresh (recap/operator.py:420-435) depends
        only on the block means of Q and K, so it is queued first: the new selection and its
        layer-wide overlap with the old partition decide which partition the new refinement
        is stored under (the host reads the overlap once the passes that use the old partition
        either way are queued, so the GPU never waits for it).  The old partition's head and coarse
        tail score the old refinement and, when the partition is kept, also give the new
        one, so one pass over every key block yields the dense output and that head.  Only
        a re-selection needs a second head pass, under the new partition."""
        if io is not None:
            query = io.shape_carrier()
        scale = self._scale(query)
        dev = query.device if io is None else io.device
        status = self.status_word(dev)
        inputs = layer.prepare(query, key, value, q_mean=True, shards=io)
        sh = inputs.shapes
        if bank.valid and not _bank_fits(bank, sh):
            # A refinement of another shape cannot be scored against this call (the
            # reference fails on the mismatch): start over as a first refresh.
            bank.release()
        revalidating = bank.valid
        selection = layer.head_partition(inputs, scale)
        overlap = None
        if revalidating:
            # the new selection's overlap with the old partition, over the whole layer; the
            # passes below use the old partition either way, so the host reads the counts only
            # after they are queued (the GPU does not wait for the host's decision)
            overlap = self._layer_overlap(selection, bank.partition)
        else:
            bank.set_partition(selection, sh.S, sh.n_video)
        full_out, full_lse, head_o, head_lse = self._dense_and_head(inputs, bank.partition, scale, status)
        context = layer.coarse_tail_context(inputs, scale)
        old_lse = bank.coarse_lse if revalidating else None
        coarse, coarse_lse, center = layer.coarse_tail_apply(
            inputs, context, bank.partition, scale, old_lse=old_lse, status=status
        )
        if bank.value is None or bank.value.shape != (sh.banks, sh.rows, sh.D):
            bank.value = torch.empty(sh.banks, sh.rows, sh.D, dtype=torch.float16, device=dev)
            bank.log_mass = torch.empty(sh.banks, sh.rows, dtype=torch.float32, device=dev)
        stats = torch.zeros(2, dtype=torch.float32, device=dev) if revalidating else None
        self._write_refinement(inputs, full_out, full_lse, head_o, head_lse, coarse, coarse_lse, bank,
                               stats, old_lse, center)
        if stats is not None:
            bank.pending_stats = stats
            bank.pending_age = self.step - bank.refreshed_at
        reselect = False
        if overlap is not None:
            # keep the old partition if the selection barely changed over the whole layer
            kept, total = (int(x) for x in overlap.cpu())
            reselect = not keep_partition(kept, total, self.config.rerank_min_overlap)
        if reselect:
            bank.set_partition(selection, sh.S, sh.n_video)
            del head_o, head_lse, coarse, coarse_lse
            head_o, head_lse = self._head(inputs, bank.partition, scale, status)
            coarse, coarse_lse, _ = layer.coarse_tail_apply(inputs, context, bank.partition, scale, status=status)
            self._write_refinement(inputs, full_out, full_lse, head_o, head_lse, coarse, coarse_lse, bank,
                                   None, None, None)
        bank.coarse_lse = coarse_lse.clone()
        bank.refreshed_at = self.step
        bank.valid = True
        self.refreshed_layers += 1
        return full_out

    def _write_refinement(self, inputs, full_out, full_lse, head_o, head_lse, coarse, coarse_lse, bank,
                          stats, old_lse, center) -> None:
        sh = inputs.shapes
        dev = full_out.device
        partials = None
        if stats is not None:
            n = int(_lib.load().recap_refresh_partials(sh.banks, sh.n_video))
            partials = torch.empty(max(n, 1), 2, dtype=torch.float32, device=dev)
        self.launches.run(
            "recap_refresh_detail", 1 + (stats is not None),
            _lib.ptr(full_out), _lib.ptr(full_lse), _lib.ptr(head_o), _lib.ptr(head_lse), _lib.ptr(coarse),
            _lib.ptr(coarse_lse), _lib.ptr(video_permutation_i32(self.layout, dev)), sh.banks, sh.S,
            sh.D, sh.n_video, video_offset(self.layout), _lib.ptr(bank.value), _lib.ptr(bank.log_mass),
            1 if stats is not None else 0, _lib.ptr(old_lse), _lib.ptr(center), _lib.ptr(partials),
            _lib.ptr(stats), _lib.stream_handle(dev),
        )

    # -- sparse ----------------------------------------------------------------------------

    @torch.no_grad()
    def _sparse(self, layer: SparseAttention, bank: DetailBank, query, key, value, io=None) -> torch.Tensor | None:
        """Head computed exactly, plus coarse tail and weighted cached refinement
        (recap/operator.py:478-527)."""
        if not bank.valid or bank.partition is None:
            raise RuntimeError("a sparse call was requested before an exact refresh")
        if io is not None:
            query = io.shape_carrier()
        scale = self._scale(query)
        dev = query.device if io is None else io.device
        status = self.status_word(dev)
        inputs = layer.prepare(query, key, value, q_mean=False, shards=io)
        sh = inputs.shapes
        if bank.partition.shape != (sh.batch, sh.heads, sh.nB, sh.nB):
            raise ValueError("the cached partition does not match this call's shape")
        context = layer.coarse_tail_context(inputs, scale)
        coarse, coarse_lse, center = layer.coarse_tail_apply(
            inputs, context, bank.partition, scale, old_lse=bank.coarse_lse, status=status
        )
        common = (_lib.ptr(inputs.q), _lib.ptr(inputs.k), _lib.ptr(inputs.v_t), _lib.ptr(bank.partition),
                  _lib.ptr(inputs.k_norm_max), sh.banks, sh.S, sh.D, sh.n_video, float(scale), _lib.ptr(coarse),
                  _lib.ptr(coarse_lse), _lib.ptr(bank.value), _lib.ptr(bank.log_mass), _lib.ptr(bank.coarse_lse),
                  _lib.ptr(center), _lib.ptr(gather_rows(self.layout, dev)))
        if io is not None:
            # the epilogue stores every row into the shard of the rank that owns its token
            self.launches.run("recap_sparse_step_ranks", 1, *common, *io.output_sinks(), _lib.ptr(status),
                              _lib.stream_handle(dev))
            return None
        out = torch.empty(sh.batch, sh.heads, sh.S, sh.D, dtype=torch.bfloat16, device=dev)
        self.launches.run("recap_sparse_step", 1, *common, _lib.ptr(out), _lib.ptr(status), _lib.stream_handle(dev))
        return out

    # -- the refinement error --------------------------------------------------------------

    def drain_validation(self) -> tuple[int, float] | None:
        """Take the scores the last refreshes left: (youngest correction age, relative RMS
        error sqrt(sum err^2 / sum ref^2) over every scored layer and rank), or None when no
        layer was scored; the pending scores are cleared (recap/operator.py:531-547)."""
        scored = [(b.pending_age, b.pending_stats) for b in self._all_banks()
                  if b.pending_stats is not None and b.pending_age is not None]
        for bank in self._all_banks():
            bank.pending_stats, bank.pending_age = None, None
        self.check_device_status()
        if not scored:
            return None
        numerator, denominator = validation_reduce(torch.stack([st for _, st in scored]).sum(dim=0),
                                                   self.process_group)
        error = math.sqrt(numerator / denominator) if denominator > 0.0 else float("inf")
        return min(int(age) for age, _ in scored), error

    def peak_bank_bytes(self) -> int:
        """Device or host bytes the stored corrections occupy (value and log-mass)."""
        return sum(t.numel() * t.element_size() for b in self._all_banks() for t in (b.value, b.log_mass)
                   if t is not None)
