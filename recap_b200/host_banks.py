"""Refinement banks in HBM where they fit, streamed from pinned host memory where not.

Drop-in for ``recap.host_banks.HostBankOperator`` (recap/host_banks.py:17-276): same
constructor, ``set_prefetch``, ``preallocate_host``, ``finish``, ``reset`` and
``peak_bank_bytes``.  The reference always keeps the refinement (``value`` fp16,
``log_mass`` fp32) in pinned host memory with two device slots.  On a 180 GB B200 this
operator first checks whether all banks fit in ``hbm_budget`` bytes (default: 40% of the
device's memory); if they do, every bank stays resident in HBM and no copy is made.  If
they do not, it streams exactly as the reference does: two device slots, the next layer
prefetched on a side stream while this layer computes, the new refinement written back on
a second stream, with events ordering the slot reuse.  Results are identical either way.

The partition and the coarse LSE reference of each layer (tens of MB) stay in HBM in
both modes.
"""

from __future__ import annotations

import torch

from .operator import REFRESH, SPARSE, Operator

_FIELDS = ("value", "log_mass")


class HostBankOperator(Operator):
    """An :class:`Operator` whose refinement is streamed from pinned host memory when the
    banks of all layers do not fit in the HBM budget."""

    def __post_init__(self) -> None:
        super().__post_init__()
        self._host: dict = {}
        self._slots: list[dict] = []
        self._slot_ready: list = [None, None]  # write-back to host finished
        self._slot_free: list = [None, None]  # compute finished reading the slot
        self._want_prefetch = True
        self._prefetch_stream = None
        self._out_stream = None
        self._prefetched = None
        self._resident: bool | None = None
        self.hbm_budget: int | None = None

    def set_prefetch(self, enabled: bool) -> None:
        """Overlap the next layer's transfer with this layer's compute."""
        self._want_prefetch = bool(enabled)

    @property
    def resident(self) -> bool | None:
        """True: banks live in HBM; False: streamed; None: not decided yet."""
        return self._resident

    # -- residency decision ---------------------------------------------------------------

    def _rows(self) -> int:
        block = int(getattr(self.config, "block_size", 128))
        return (self.layout.video_tokens // block) * block

    def _decide(self, n_banks: int, dim: int, device) -> bool:
        if self._resident is None:
            per_layer = n_banks * self._rows() * (dim * 2 + 4)
            total = per_layer * sum(len(row) for row in self.layers)
            budget = self.hbm_budget
            if budget is None:
                if torch.cuda.is_available():
                    budget = int(0.4 * torch.cuda.get_device_properties(device).total_memory)
                else:
                    budget = 0
            self._resident = total <= budget
        return self._resident

    # -- device slots ---------------------------------------------------------------------

    def _alloc_slots(self, n_banks: int, rows: int, dim: int, device) -> None:
        self._slots = []
        for _ in range(2 if self._want_prefetch else 1):
            self._slots.append({
                "value": torch.empty((n_banks, rows, dim), dtype=torch.float16, device=device),
                "log_mass": torch.empty((n_banks, rows), dtype=torch.float32, device=device),
            })
        if self._want_prefetch and self._prefetch_stream is None:
            self._prefetch_stream = torch.cuda.Stream(device=device)
        if self._out_stream is None:
            self._out_stream = torch.cuda.Stream(device=device)

    def _ensure_slots(self, query: torch.Tensor) -> None:
        b, h, _, dim = query.shape
        n_banks, rows = b * h, self._rows()
        if self._slots and self._slots[0]["value"].shape == (n_banks, rows, dim):
            return
        self._alloc_slots(n_banks, rows, dim, query.device)

    @staticmethod
    def _new_host_bank(n_banks: int, rows: int, dim: int) -> dict:
        return {
            "value": torch.empty((n_banks, rows, dim), dtype=torch.float16).pin_memory(),
            "log_mass": torch.empty((n_banks, rows), dtype=torch.float32).pin_memory(),
        }

    def _host_bank(self, key_id) -> dict:
        existing = self._host.get(key_id)
        if existing is not None:
            return existing
        n_banks, rows, dim = self._slots[0]["value"].shape
        made = self._new_host_bank(n_banks, rows, dim)
        self._host[key_id] = made
        return made

    def preallocate_host(self, n_layers: int, n_banks: int, dim: int) -> int:
        """Decide residency; when streaming, allocate all host memory and the device slots.
        Returns the bytes held by the refinement (host bytes when streaming)."""
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else None
        if self._decide(n_banks, dim, device):
            return 0
        rows = self._rows()
        for stream in range(self.n_streams):
            for layer in range(min(n_layers, len(self.layers[stream]))):
                key_id = (stream, layer)
                if key_id not in self._host:
                    self._host[key_id] = self._new_host_bank(n_banks, rows, dim)
        if device is not None and not self._slots:
            self._alloc_slots(n_banks, rows, dim, device)
        return self.peak_bank_bytes()

    @staticmethod
    def _copy(dst: dict, src: dict, *, non_blocking: bool) -> None:
        for name in _FIELDS:
            if dst.get(name) is not None and src.get(name) is not None:
                dst[name].copy_(src[name], non_blocking=non_blocking)

    # -- dispatch -------------------------------------------------------------------------

    @torch.no_grad()
    def attend(self, layer_index: int, query, key, value):
        if self.kind not in (REFRESH, SPARSE):
            return super().attend(layer_index, query, key, value)
        b, h, _, dim = query.shape
        if self._decide(b * h, dim, query.device):
            return super().attend(layer_index, query, key, value)

        bank = self.banks[self.stream][layer_index]
        self._ensure_slots(query)
        index = layer_index % len(self._slots)
        slot = self._slots[index]
        key_id = (self.stream, layer_index)
        host = self._host.get(key_id)
        if host is not None and host["value"].shape != slot["value"].shape:
            self._host.pop(key_id)
            host = None
        pending = self._slot_ready[index]
        if pending is not None:
            torch.cuda.current_stream().wait_event(pending)
            self._slot_ready[index] = None
        if self.kind == SPARSE:
            if host is None or not bank.valid:
                raise RuntimeError("a sparse call was requested before an exact refresh")
            self._stage_in(key_id, slot)
        elif bank.valid and host is not None:
            self._stage_in(key_id, slot)  # the refresh scores the old refinement
        bank.value, bank.log_mass = slot["value"], slot["log_mass"]
        try:
            out = super().attend(layer_index, query, key, value)
        finally:
            if self.kind == REFRESH:
                self._stage_out(key_id, slot, index)
            released = torch.cuda.Event()
            released.record()
            self._slot_free[index] = released
            bank.value = bank.log_mass = None
        return out

    def _stage_in(self, key_id, slot: dict) -> None:
        host = self._host[key_id]
        if self._prefetched == key_id and self._prefetch_stream is not None:
            torch.cuda.current_stream().wait_stream(self._prefetch_stream)
            self._prefetched = None
        else:
            self._copy(slot, host, non_blocking=True)
        self._maybe_prefetch(key_id)

    def _maybe_prefetch(self, key_id) -> None:
        """Copy the next layer's refinement while this layer computes."""
        if self._prefetch_stream is None:
            return
        stream, layer = key_id
        nxt = (stream, layer + 1)
        if nxt not in self._host:
            return
        index = (layer + 1) % len(self._slots)
        if self._slot_ready[index] is not None:
            return  # still being written back
        with torch.cuda.stream(self._prefetch_stream):
            released = self._slot_free[index]
            if released is not None:
                self._prefetch_stream.wait_event(released)
            self._copy(self._slots[index], self._host[nxt], non_blocking=True)
        self._prefetched = nxt

    def _stage_out(self, key_id, slot: dict, index: int) -> None:
        """Copy the new refinement to host memory on the write-back stream."""
        host = self._host_bank(key_id)
        written = torch.cuda.Event()
        written.record()
        with torch.cuda.stream(self._out_stream):
            self._out_stream.wait_event(written)
            self._copy(host, slot, non_blocking=True)
            event = torch.cuda.Event()
            event.record()
        self._slot_ready[index] = event

    # -- bookkeeping ----------------------------------------------------------------------

    def finish(self) -> None:
        """Wait for all transfers in flight."""
        for events in (self._slot_ready, self._slot_free):
            for event in events:
                if event is not None:
                    event.synchronize()
        if self._prefetch_stream is not None:
            self._prefetch_stream.synchronize()
        if self._out_stream is not None:
            self._out_stream.synchronize()
        self._slot_ready = [None, None]
        self._slot_free = [None, None]
        self._prefetched = None

    def reset(self) -> None:
        self.finish()
        super().reset()

    def __del__(self):  # pragma: no cover - teardown path
        try:
            self.finish()
        except Exception:
            pass

    def peak_bank_bytes(self) -> int:
        """Bytes held by the refinement: host bytes when streaming, else device bytes."""
        if self._resident is False:
            return sum(
                t.numel() * t.element_size() for bank in self._host.values() for t in bank.values() if t is not None
            )
        return super().peak_bank_bytes()
