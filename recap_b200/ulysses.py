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
