"""Refinement banks in HBM where they fit, streamed through a ring of device slots where not.

Drop-in for ``recap.host_banks.HostBankOperator`` (recap/host_banks.py:17-97 is the API
kept: ``build``, ``set_prefetch``, ``preallocate_host``, ``finish``, ``reset``,
``peak_bank_bytes``).

Residency first.  A B200 has 180 GB of HBM; a 60-layer HunyuanVideo-720p stack needs
45 GB of refinement at one GPU and 5.6 GB per GPU at eight.  So the operator first asks
whether the banks of every layer fit in ``hbm_budget`` bytes (default: 40% of the
device's memory).  If they do, each layer's bank is an ordinary device tensor and no copy
is ever made.

Streaming otherwise.  The refinement (``value`` fp16, ``log_mass`` fp32) of every
(stream, layer) lives in pinned host memory, and a small ring of device slots caches the
banks in use:

* a slot remembers which bank it holds and carries three events: ``loaded`` (its
  host-to-device copy finished), ``released`` (the last kernel reading or writing it
  finished) and ``saved`` (its device-to-host write-back finished);
* a call takes the slot that already holds its bank (a hit, e.g. a prefetch) or else the
  least recently used slot, whose copy-in then waits on that slot's ``released`` and
  ``saved`` events on the copy-in stream; the compute stream waits on ``loaded``;
* after a REFRESH call the new refinement goes back to host memory on the write-back
  stream, which waits for the compute stream's event; after any call the slot's
  ``released`` event is recorded;
* with prefetch on, every call also starts the copy-in of the bank it expects next
  ((stream, layer + 1), which the step loop calls next) into another slot, so the
  transfer runs on the copy engine while this layer computes.

Only the refinement streams.  Each layer's partition (tens of MB) and coarse-LSE
reference stay in HBM in both modes.  The copies are exact, so the streamed operator's
results equal the resident operator's bit for bit.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .operator import REFRESH, SPARSE, Operator


@dataclass
class _Slot:
    """One device slot of the ring."""

    value: torch.Tensor
    log_mass: torch.Tensor
    key: tuple | None = None          # (stream, layer) whose refinement it holds
    valid: bool = False               # holds that bank's current refinement
    last_use: int = -1                # call counter at its last use (LRU order)
    loaded: torch.cuda.Event | None = None
    released: torch.cuda.Event | None = None
    saved: torch.cuda.Event | None = None

    def tensors(self) -> dict:
        return {"value": self.value, "log_mass": self.log_mass}


class HostBankOperator(Operator):
    """An :class:`Operator` whose refinement is streamed from pinned host memory when the
    banks of all layers do not fit in the HBM budget."""

    #: device slots of the ring when streaming (two: the layer in use and the next one)
    ring_slots: int = 2

    def __post_init__(self) -> None:
        super().__post_init__()
        self.hbm_budget: int | None = None
        self._prefetch = True
        self._resident: bool | None = None
        self._host: dict[tuple, dict] = {}
        self._ring: list[_Slot] = []
        self._calls = 0
        self._copy_in: torch.cuda.Stream | None = None
        self._copy_out: torch.cuda.Stream | None = None

    # -- the reference API ----------------------------------------------------------------

    def set_prefetch(self, enabled: bool) -> None:
        """Overlap the next layer's transfer with this layer's compute."""
        self._prefetch = bool(enabled)

    @property
    def resident(self) -> bool | None:
        """True: banks live in HBM; False: streamed; None: not decided yet."""
        return self._resident

    def preallocate_host(self, n_layers: int, n_banks: int, dim: int) -> int:
        """Decide residency; when streaming, allocate every host bank and the device ring.
        Returns the bytes the refinement holds (host bytes when streaming, 0 when the
        banks will live in HBM and nothing is allocated yet)."""
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else None
        if self._choose_residency(n_banks, dim, device):
            return 0
        for stream in range(self.n_streams):
            for layer in range(min(n_layers, len(self.layers[stream]))):
                self._host_bank((stream, layer), n_banks, dim)
        if device is not None:
            self._ensure_ring(n_banks, dim, device)
        return self.peak_bank_bytes()

    def finish(self) -> None:
        """Wait for every transfer in flight."""
        for slot in self._ring:
            for ev in (slot.loaded, slot.saved, slot.released):
                if ev is not None:
                    ev.synchronize()
        for st in (self._copy_in, self._copy_out):
            if st is not None:
                st.synchronize()

    def reset(self) -> None:
        self.finish()
        for slot in self._ring:
            slot.key, slot.valid, slot.last_use = None, False, -1
        super().reset()

    def peak_bank_bytes(self) -> int:
        """Bytes held by the refinement: host bytes when streaming, else device bytes."""
        if self._resident is False:
            return sum(t.numel() * t.element_size() for bank in self._host.values() for t in bank.values())
        return super().peak_bank_bytes()

    def __del__(self):  # pragma: no cover - interpreter teardown
        try:
            self.finish()
        except Exception:
            pass

    # -- residency ------------------------------------------------------------------------

    def _rows(self) -> int:
        block = int(getattr(self.config, "block_size", 128))
        return (self.layout.video_tokens // block) * block

    def _choose_residency(self, n_banks: int, dim: int, device) -> bool:
        if self._resident is None:
            n_layers = sum(len(row) for row in self.layers)
            need = n_layers * n_banks * self._rows() * (2 * dim + 4)
            budget = self.hbm_budget
            if budget is None:
                budget = int(0.4 * torch.cuda.get_device_properties(device).total_memory) if device is not None else 0
            self._resident = need <= budget
        return self._resident

    # -- host banks and the ring ----------------------------------------------------------

    def _host_bank(self, key: tuple, n_banks: int, dim: int) -> dict:
        rows = self._rows()
        bank = self._host.get(key)
        if bank is None or tuple(bank["value"].shape) != (n_banks, rows, dim):
            bank = {
                "value": torch.empty(n_banks, rows, dim, dtype=torch.float16).pin_memory(),
                "log_mass": torch.empty(n_banks, rows, dtype=torch.float32).pin_memory(),
            }
            self._host[key] = bank
        return bank

    def _ensure_ring(self, n_banks: int, dim: int, device) -> None:
        rows = self._rows()
        if self._ring and tuple(self._ring[0].value.shape) == (n_banks, rows, dim):
            return
        self.finish()
        count = max(2, int(self.ring_slots)) if self._prefetch else 1
        self._ring = [_Slot(value=torch.empty(n_banks, rows, dim, dtype=torch.float16, device=device),
                            log_mass=torch.empty(n_banks, rows, dtype=torch.float32, device=device))
                      for _ in range(count)]
        if self._copy_in is None:
            self._copy_in = torch.cuda.Stream(device=device)
            self._copy_out = torch.cuda.Stream(device=device)

    def _slot_of(self, key: tuple) -> _Slot | None:
        for slot in self._ring:
            if slot.key == key and slot.valid:
                return slot
        return None

    def _victim(self, avoid: _Slot | None = None) -> _Slot:
        free = [s for s in self._ring if s is not avoid]
        return min(free, key=lambda s: s.last_use)

    def _fill(self, slot: _Slot, key: tuple) -> None:
        """Copy host bank ``key`` into ``slot`` on the copy-in stream."""
        host = self._host[key]
        st = self._copy_in
        with torch.cuda.stream(st):
            for ev in (slot.released, slot.saved):
                if ev is not None:
                    st.wait_event(ev)
            for name, dst in slot.tensors().items():
                dst.copy_(host[name], non_blocking=True)
            slot.loaded = torch.cuda.Event()
            slot.loaded.record(st)
        slot.key, slot.valid = key, True

    def _take(self, key: tuple, load: bool) -> _Slot:
        """The slot for bank ``key``; with ``load``, holding its host refinement."""
        slot = self._slot_of(key)
        if slot is None:
            slot = self._victim()
            if load:
                self._fill(slot, key)
            else:
                slot.key, slot.valid, slot.loaded = key, True, None
                comp = torch.cuda.current_stream()
                for ev in (slot.released, slot.saved):
                    if ev is not None:
                        comp.wait_event(ev)  # the kernels overwrite it: earlier readers first
        if slot.loaded is not None:
            torch.cuda.current_stream().wait_event(slot.loaded)
        self._calls += 1
        slot.last_use = self._calls
        return slot

    def _prefetch_next(self, key: tuple, current: _Slot) -> None:
        stream, layer = key
        nxt = (stream, layer + 1)
        if not self._prefetch or len(self._ring) < 2 or nxt not in self._host:
            return
        if layer + 1 >= len(self.banks[stream]):
            return
        if self._slot_of(nxt) is not None or not self.banks[stream][layer + 1].valid:
            return
        self._fill(self._victim(avoid=current), nxt)

    def _write_back(self, slot: _Slot, key: tuple) -> None:
        host = self._host[key]
        written = torch.cuda.Event()
        written.record(torch.cuda.current_stream())
        st = self._copy_out
        with torch.cuda.stream(st):
            st.wait_event(written)
            for name, src in slot.tensors().items():
                host[name].copy_(src, non_blocking=True)
            slot.saved = torch.cuda.Event()
            slot.saved.record(st)

    # -- dispatch -------------------------------------------------------------------------

    @torch.no_grad()
    def attend(self, layer_index: int, query, key, value):
        if self.kind not in (REFRESH, SPARSE):
            return super().attend(layer_index, query, key, value)
        b, h, _, dim = query.shape
        if self._choose_residency(b * h, dim, query.device):
            return super().attend(layer_index, query, key, value)

        ident = (self.stream, layer_index)
        bank = self.banks[self.stream][layer_index]
        self._ensure_ring(b * h, dim, query.device)
        host = self._host.get(ident)
        if host is not None and tuple(host["value"].shape) != tuple(self._ring[0].value.shape):
            del self._host[ident]  # another shape: the old refinement cannot be used
            host = None
        if self.kind == SPARSE and (host is None or not bank.valid):
            raise RuntimeError("a sparse call was requested before an exact refresh")
        if host is None:
            self._host_bank(ident, b * h, dim)
        # a SPARSE step and a revalidating REFRESH read the stored refinement
        slot = self._take(ident, load=bank.valid)
        self._prefetch_next(ident, slot)
        bank.value, bank.log_mass = slot.value, slot.log_mass
        try:
            out = super().attend(layer_index, query, key, value)
        finally:
            if self.kind == REFRESH:
                self._write_back(slot, ident)
            slot.released = torch.cuda.Event()
            slot.released.record(torch.cuda.current_stream())
            bank.value = bank.log_mass = None
        return out
