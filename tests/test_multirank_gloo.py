"""Head sharding on CPU ranks (gloo, world size 2): the layer-wide re-selection decision
and the validation sums give every rank the answer of the single-process operator, and a
rank that leaves before a collective makes the other's collective fail within its
timeout instead of hanging."""

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 30.0):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _decision_worker(rank: int, world: int, port: int, results):
    from recap_b200.operator import keep_partition, layer_counts_reduce, validation_reduce

    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(0)
        heads, nb = 6, 12
        new = torch.rand(heads, nb, nb, generator=g) < 0.3
        old = new.clone()
        flip = torch.rand(heads, nb, nb, generator=g) < 0.08
        old ^= flip
        stats = torch.rand(heads, 2, generator=g, dtype=torch.float64)
        lo, hi = rank * heads // world, (rank + 1) * heads // world
        counts = torch.tensor([int((new[lo:hi] & old[lo:hi]).sum()), int(new[lo:hi].sum())], dtype=torch.int64)
        kept, total = layer_counts_reduce(counts, dist.group.WORLD)
        num, den = validation_reduce(stats[lo:hi].sum(0), dist.group.WORLD)
        results[rank] = (kept, total, keep_partition(kept, total, 0.95), num, den)
    finally:
        dist.destroy_process_group()


def _leaving_worker(rank: int, world: int, port: int, results):
    _init(rank, world, port, timeout_s=5.0)
    if rank == 1:
        results[rank] = "left"
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        t = torch.ones(2)
        dist.all_reduce(t)
        results[rank] = "no error"
    except Exception as e:  # gloo reports the lost peer or the timeout
        results[rank] = f"error: {type(e).__name__}"


def test_layer_decision_and_validation_match_single_process():
    from recap_b200.operator import keep_partition

    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    port = _port()
    mp.start_processes(_decision_worker, args=(2, port, results), nprocs=2, start_method="spawn", join=True)
    g = torch.Generator().manual_seed(0)
    new = torch.rand(6, 12, 12, generator=g) < 0.3
    old = new.clone()
    old ^= torch.rand(6, 12, 12, generator=g) < 0.08
    stats = torch.rand(6, 2, generator=g, dtype=torch.float64)
    kept, total = int((new & old).sum()), int(new.sum())
    expect = (kept, total, keep_partition(kept, total, 0.95))
    for r in range(2):
        assert tuple(results[r][:3]) == expect
        assert results[r][3] == pytest.approx(float(stats[:, 0].sum()), rel=1e-12)
        assert results[r][4] == pytest.approx(float(stats[:, 1].sum()), rel=1e-12)


def test_rank_leaving_makes_peer_collective_fail_not_hang():
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    port = _port()
    ctx = mp.start_processes(_leaving_worker, args=(2, port, results), nprocs=2, start_method="spawn", join=False)
    for p in ctx.processes:
        p.join(timeout=90)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung on a collective"
    assert results.get(1) == "left"
    assert str(results.get(0, "")).startswith("error"), results.get(0)


def _global_qkv(S: int, H: int, d: int) -> torch.Tensor:
    """[S, 3, H, d] with every element naming its (token, tensor, head, column)."""
    t = torch.arange(S).view(S, 1, 1, 1) * 1000.0
    i = torch.arange(3).view(1, 3, 1, 1) * 100.0
    h = torch.arange(H).view(1, 1, H, 1) * 10.0
    c = torch.arange(d).view(1, 1, 1, d) * 1.0
    return t + i + h + c


def _ulysses_worker(rank: int, world: int, port: int, results):
    from recap_b200.ulysses import check_split, heads_to_seq, seq_to_heads

    _init(rank, world, port)
    try:
        S, H, d = 12, 4, 3
        s, h = check_split(S, H, world)
        full = _global_qkv(S, H, d)
        mine = full[rank * s:(rank + 1) * s].contiguous()  # this rank's tokens, every head
        q, k, v = seq_to_heads(mine, world, dist.group.WORLD)
        # every token of this rank's heads, as the operator's [1, h, S, d]
        ok = all(torch.equal(x[0], full[:, i, rank * h:(rank + 1) * h].permute(1, 0, 2))
                 for i, x in enumerate((q, k, v)))
        # stand-in attention output: distinct per (head, token, column)
        out = (q * 2.0 + 1.0).contiguous()
        back = heads_to_seq(out, world, dist.group.WORLD)  # [s, H d]
        expect = (full[rank * s:(rank + 1) * s, 0] * 2.0 + 1.0).reshape(s, H * d)
        results[rank] = (ok, bool(torch.equal(back, expect)), tuple(q.shape), tuple(back.shape))
    finally:
        dist.destroy_process_group()


def test_ulysses_layout_switch_round_trip():
    """The sequence -> head switch hands each rank every token of its heads in token order,
    and the head -> sequence switch returns each rank its own tokens of every head in the
    global head order (world size 2, gloo all_to_all_single on CPU)."""
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    port = _port()
    mp.start_processes(_ulysses_worker, args=(2, port, results), nprocs=2, start_method="spawn", join=True)
    for r in range(2):
        assert results[r] == (True, True, (1, 2, 12, 3), (6, 12)), results[r]


def test_ulysses_single_rank_is_identity_and_rejects_uneven_splits():
    from recap_b200.ulysses import check_split, heads_to_seq, seq_to_heads

    full = _global_qkv(10, 4, 3)
    q, k, v = seq_to_heads(full, 1)
    assert torch.equal(q[0], full[:, 0].permute(1, 0, 2))
    assert torch.equal(heads_to_seq(v.contiguous(), 1), full[:, 2].reshape(10, 12))
    with pytest.raises(ValueError):
        check_split(10, 4, 4)
    with pytest.raises(ValueError):
        check_split(12, 6, 4)
