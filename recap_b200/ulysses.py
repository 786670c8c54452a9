"""Ulysses sequence-to-head layout switch for the multi-GPU transformer stack.

A DiT block holds its activations sharded by sequence: rank p of P owns tokens
``[p S/P, (p+1) S/P)`` of the hidden states ``[S, hidden]``.  The attention of a layer
needs every token of a head, so the layer's Q/K/V projection output goes through one
all-to-all that hands each rank all tokens of its ``H/P`` heads (sequence -> head), the
operator attends on those heads, and a second all-to-all returns every rank its own
tokens of all heads (head -> sequence) before the output projection.  This is the
layout switch RECAP's multi-GPU runs use around ``Operator.attend``: the operator itself
is head-parallel with no collective inside a SPARSE step.

The exchange is ``torch.distributed.all_to_all_single`` (NCCL over NVLink on B200, gloo
on CPU): chunk ``p`` of the send buffer goes to rank ``p`` and chunk ``p`` of the receive
buffer comes from rank ``p``.  Sequence shards are contiguous and ordered by rank, so the
receive buffer of the sequence -> head switch is already in token order.

Shapes (``s = S / P`` tokens per rank, ``h = H / P`` heads per rank):
    seq_to_heads:  qkv ``[s, 3, H, d]``  ->  q, k, v ``[1, h, S, d]`` (views, d contiguous)
    heads_to_seq:  out ``[1, h, S, d]``  ->  ``[s, H d]`` (heads in global order)
"""

from __future__ import annotations

import torch


def check_split(seq: int, heads: int, world: int) -> tuple[int, int]:
    """Tokens and heads per rank; the Ulysses switch needs both to divide evenly."""
    if world < 1 or seq % world or heads % world:
        raise ValueError(f"sequence {seq} and heads {heads} must both split evenly over {world} ranks")
    return seq // world, heads // world


def _exchange(send: torch.Tensor, group) -> torch.Tensor:
    import torch.distributed as dist

    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv


def seq_to_heads(qkv: torch.Tensor, world: int, group=None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``[s, 3, H, d]`` projections of this rank's tokens -> Q, K, V ``[1, H/P, S, d]`` of
    this rank's heads over the whole sequence.

    Send chunk p holds this rank's tokens of head group p (heads ``[p h, (p+1) h)``);
    receive chunk p holds rank p's tokens of this rank's head group, so the received
    ``[P, s, 3, h, d]`` is ``[S, 3, h, d]`` in token order."""
    s, three, H, d = qkv.shape
    if three != 3 or H % world:
        raise ValueError("qkv must be [tokens, 3, heads, dim] with heads divisible by the world size")
    h = H // world
    if world == 1:
        full = qkv  # nothing to exchange: the heads are views of the projection output
    else:
        send = qkv.view(s, 3, world, h, d).permute(2, 0, 1, 3, 4).contiguous()
        full = _exchange(send, group).view(world * s, 3, h, d)
    q, k, v = (full[:, i].permute(1, 0, 2).unsqueeze(0) for i in range(3))
    return q, k, v


def heads_to_seq(out: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """``[1, h, S, d]`` attention output of this rank's heads -> ``[s, H d]`` of this rank's
    tokens over all heads (the operand of the output projection).

    Send chunk p holds tokens ``[p s, (p+1) s)`` of this rank's heads; receive chunk p
    holds this rank's tokens of head group p."""
    _, h, S, d = out.shape
    if S % world:
        raise ValueError("the sequence must split evenly over the world size")
    s = S // world
    if world == 1:
        return out[0].permute(1, 0, 2).reshape(S, h * d)
    send = out[0].reshape(h, world, s, d).permute(1, 2, 0, 3).contiguous()  # [P, s, h, d]
    recv = _exchange(send, group)  # [P (head group), s, h, d]
    return recv.permute(1, 0, 2, 3).reshape(s, world * h * d)


# ----------------------------------------------------------------------------- in place over NVLink


class PeerBuffer:
    """``nbytes`` of device memory on every rank of ``group`` (one process per GPU), each rank
    holding the address of every rank's buffer: allocated by ``recap_peer_alloc`` and shared
    by CUDA IPC handles exchanged over the process group.  ``close()`` (collective) releases
    the mappings and the memory."""

    def __init__(self, nbytes: int, group, device: torch.device):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        lib = _lib.load()
        self.device = device
        self.nbytes = int(nbytes)
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        own = ctypes.c_void_p()
        _lib.check(lib.recap_peer_alloc(self.nbytes, ctypes.byref(own)), "recap_peer_alloc")
        handle = ctypes.create_string_buffer(lib.recap_peer_handle_bytes())
        _lib.check(lib.recap_peer_export(own, handle), "recap_peer_export")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.ptrs: list[int] = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.ptrs.append(int(own.value))
                continue
            p = ctypes.c_void_p()
            _lib.check(lib.recap_peer_import(ctypes.create_string_buffer(h, len(h)), ctypes.byref(p)),
                       "recap_peer_import")
            self.ptrs.append(int(p.value))

    def local(self, shape, dtype: torch.dtype) -> torch.Tensor:
        """A tensor over this rank's buffer (no copy)."""
        return _tensor_at(self.ptrs[self.rank], shape, dtype, self.device)

    def close(self) -> None:
        import torch.distributed as dist

        from . import _lib

        if not self.ptrs:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank reads or writes another's buffer any more
        lib = _lib.load()
        for q, p in enumerate(self.ptrs):
            if q != self.rank:
                _lib.check(lib.recap_peer_close(p), "recap_peer_close")
        dist.barrier(group=self.group)  # every mapping of this rank's buffer is closed
        _lib.check(lib.recap_peer_free(self.ptrs[self.rank]), "recap_peer_free")
        self.ptrs = []


class _CudaView:
    def __init__(self, ptr: int, numel: int):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _tensor_at(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A tensor of 2-byte elements at a device address this process can reach (its own or an
    imported peer buffer)."""
    if torch.empty(0, dtype=dtype).element_size() != 2:
        raise ValueError("2-byte element types only")
    numel = 1
    for n in shape:
        numel *= int(n)
    with torch.cuda.device(device):
        flat = torch.as_tensor(_CudaView(ptr, numel), device=device)
    return flat.view(dtype).view(*shape)


class ShardedIO:
    """The operands of one sequence-parallel attention call, left where the ranks hold them:
    rank q's projection output ``[s, 3, H, d]`` (bf16) in ``qkv.ptrs[q]`` and its attention
    output ``[s, H, d]`` in ``out.ptrs[q]``.  This rank attends on heads
    ``[head0, head0 + heads)``: the layout pass reads their Q, K, V rows from every rank's
    projection buffer, and the SPARSE step's epilogue stores every output row into the
    buffer of the rank that owns the token."""

    def __init__(self, qkv: PeerBuffer, out: PeerBuffer, total_heads: int, dim: int, seq: int,
                 recv: PeerBuffer | None = None):
        """``recv`` (push mode): each rank's receive buffer ``[S, 3, H/P, d]`` of its heads'
        projections; ``push`` writes every rank's rows into it with copy-engine peer writes
        and the layout pass then reads it locally.  Without it the layout pass reads the
        ranks' projection buffers ``qkv`` in place."""
        world, rank = out.world, out.rank
        self.tokens_per_rank, self.heads = check_split(seq, total_heads, world)
        self.qkv, self.out = qkv, out
        self.world, self.rank = world, rank
        self.total_heads, self.dim, self.seq = total_heads, dim, seq
        self.head0 = rank * self.heads
        self.device = out.device
        self.recv = recv
        need_qkv = self.tokens_per_rank * 3 * total_heads * dim * 2
        need_out = self.tokens_per_rank * total_heads * dim * 2
        if (qkv is not None and qkv.nbytes < need_qkv) or out.nbytes < need_out:
            raise ValueError("peer buffers smaller than the token shards")
        if recv is not None and recv.nbytes < seq * 3 * self.heads * dim * 2:
            raise ValueError("receive buffer smaller than the heads' projections")

    def shape_carrier(self) -> torch.Tensor:
        """A shape-only ``[1, heads, S, d]`` tensor (the layer call's geometry)."""
        return torch.empty(1, self.heads, self.seq, self.dim, device="meta")

    def local_qkv(self) -> torch.Tensor:
        return self.qkv.local((self.tokens_per_rank, 3, self.total_heads, self.dim), torch.bfloat16)

    def local_out(self) -> torch.Tensor:
        return self.out.local((self.tokens_per_rank, self.total_heads * self.dim), torch.bfloat16)

    def push(self, qkv_local: torch.Tensor) -> None:
        """Push mode: write this rank's ``[s, 3, H, d]`` projections of every head group into
        the receive buffer of the rank that owns it, at this rank's token range: one kernel of
        16-byte peer stores over NVLink (``recap_push_heads``)."""
        import ctypes

        from . import _lib

        s, H, d = self.tokens_per_rank, self.total_heads, self.dim
        if tuple(qkv_local.shape) != (s, 3, H, d) or not qkv_local.is_contiguous():
            raise ValueError("push takes this rank's contiguous [s, 3, H, d] projections")
        dst = (ctypes.c_void_p * self.world)(*self.recv.ptrs)
        _lib.call("recap_push_heads", _lib.ptr(qkv_local), s, H, d, self.rank, self.world, dst,
                  _lib.stream_handle(qkv_local.device))

    def gather_call(self):
        """The layout pass's entry point and its leading arguments (up to the head count)."""
        import ctypes

        if self.recv is not None:
            h, d = self.heads, self.dim
            base = self.recv.ptrs[self.rank]
            row = 3 * h * d
            strides = (ctypes.c_int64 * 9)(*([self.seq * row, d, row] * 3))
            return ("recap_layout_gather", base, base + h * d * 2, base + 2 * h * d * 2, strides, 1, self.heads)
        qr, kr, vr, n, tpr, strides = self.gather_sources()
        return ("recap_layout_gather_ranks", qr, kr, vr, n, tpr, strides, self.heads)

    def gather_sources(self):
        """Arguments of ``recap_layout_gather_ranks``: per-rank addresses of head ``head0`` of
        Q, K and V, the rank count, tokens per rank and the element strides."""
        import ctypes

        H, d = self.total_heads, self.dim
        arrs = []
        for t in range(3):
            off = (t * H + self.head0) * d * 2
            arrs.append((ctypes.c_void_p * self.world)(*[p + off for p in self.qkv.ptrs]))
        row = 3 * H * d
        strides = (ctypes.c_int64 * 9)(*([self.seq * row, d, row] * 3))
        return arrs[0], arrs[1], arrs[2], self.world, self.tokens_per_rank, strides

    def output_sinks(self):
        """Arguments of the ``*_ranks`` attention passes: per-rank addresses of head
        ``head0`` of token 0, rank count, tokens per rank, bank and row strides."""
        import ctypes

        d = self.dim
        ptrs = (ctypes.c_void_p * self.world)(*[p + self.head0 * d * 2 for p in self.out.ptrs])
        return ptrs, self.world, self.tokens_per_rank, d, self.total_heads * d

    def scatter_output(self, out: torch.Tensor) -> None:
        """Store a contiguous ``[1, heads, S, d]`` attention output computed locally into the
        ranks' output buffers (copy-engine peer copies over NVLink)."""
        from . import _lib

        if not out.is_contiguous() or tuple(out.shape) != (1, self.heads, self.seq, self.dim):
            raise ValueError("scatter_output takes this rank's contiguous [1, heads, S, d] output")
        ptrs, n, tpr, bank_stride, row_stride = self.output_sinks()
        _lib.call("recap_scatter_rows", _lib.ptr(out), self.heads, self.seq, self.dim, ptrs, n, tpr, bank_stride,
                  row_stride, _lib.stream_handle(out.device))
