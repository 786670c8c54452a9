"""The Ulysses exchange across real ranks (two GPUs, one process each, NCCL, CUDA IPC buffers):
one attention layer of a sequence-parallel stack through REFRESH -> SPARSE -> revalidating
REFRESH -> SPARSE, with the exchange done three ways - peer stores into the owners' receive
buffers (push), the layout pass reading the ranks' projections in place (p2p), and NCCL
all_to_all_single around ``Operator.attend`` (nccl).  The same kernels see the same values
in every mode, so the layer outputs agree bit for bit when the first refresh's eigen-solve
(cuSOLVER, run once per mode) repeats exactly; the test asserts the parity tolerance
(max-abs 2e-2) and prints whether the bits agree.  Skipped with fewer than two GPUs."""

import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

H, D, GRID, TEXT = 4, 128, (4, 8, 16), 64  # 512 video tokens + 64 text tokens, 4 heads of 128


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_outputs(mode: str, world: int, rank: int, group, dev, xs, w_qkv):
    """This rank's [s, H D] attention output of each step (before the output projection)."""
    import torch.distributed as dist

    from recap_b200 import REFRESH, SPARSE, Operator, OperatorConfig
    from recap_b200.sparse import Layout, SparseGeometry, hilbert_permutation
    from recap_b200.ulysses import PeerBuffer, ShardedIO, heads_to_seq, seq_to_heads

    layout = Layout.from_permutation(hilbert_permutation(GRID), text_tokens=TEXT, text_first=False)
    op = Operator.build(OperatorConfig(head_density=0.3), SparseGeometry.build(layout, 128), n_layers=1,
                        process_group=group)
    S = layout.video_tokens + TEXT
    s = S // world
    flag = torch.zeros(1, device=dev)
    peers = []
    io = None
    if mode in ("push", "p2p"):
        out = PeerBuffer(s * H * D * 2, group, dev)
        peers.append(out)
        if mode == "push":
            recv = PeerBuffer(S * 3 * (H // world) * D * 2, group, dev)
            peers.append(recv)
            io = ShardedIO(None, out, total_heads=H, dim=D, seq=S, recv=recv)
        else:
            qkvb = PeerBuffer(s * 3 * H * D * 2, group, dev)
            peers.append(qkvb)
            io = ShardedIO(qkvb, out, total_heads=H, dim=D, seq=S)
    got = []
    for step, (kind, x) in enumerate(zip((REFRESH, SPARSE, REFRESH, SPARSE), xs)):
        op.begin_step(step, kind)
        qkv = (x @ w_qkv).view(s, 3, H, D)
        if mode == "nccl":
            q, k, v = seq_to_heads(qkv, world, group)
            y = heads_to_seq(op.attend(0, q, k, v), world, group)
        else:
            if mode == "push":
                io.push(qkv.contiguous())
            else:
                io.local_qkv().copy_(qkv)
            dist.all_reduce(flag, group=group)
            op.attend_sharded(0, io)
            dist.all_reduce(flag, group=group)
            y = io.local_out().clone()
        got.append(y.cpu())
    op.check_device_status()
    torch.cuda.synchronize()
    for p in peers:
        p.close()
    return got


def _worker(rank: int, world: int, port: int, results):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=dev)
    try:
        from recap_b200.sparse import hilbert_permutation

        S = len(hilbert_permutation(GRID)) + TEXT
        s = S // world
        g = torch.Generator().manual_seed(11)
        hidden = H * D
        x0 = torch.randn(S, hidden, generator=g)
        xs = [x0 + 0.05 * i * torch.randn(S, hidden, generator=g) for i in range(4)]
        xs = [x[rank * s:(rank + 1) * s].to(torch.bfloat16).to(dev) for x in xs]
        w_qkv = (torch.randn(hidden, 3 * hidden, generator=g) / hidden ** 0.5).to(torch.bfloat16).to(dev)
        outs = {m: _layer_outputs(m, world, rank, dist.group.WORLD, dev, xs, w_qkv) for m in ("nccl", "push", "p2p")}
        ok = {m: all(torch.equal(a, b) for a, b in zip(outs[m], outs["nccl"])) for m in ("push", "p2p")}
        diff = {m: max(float((a.float() - b.float()).abs().max()) for a, b in zip(outs[m], outs["nccl"]))
                for m in ("push", "p2p")}
        finite = all(bool(torch.isfinite(t.float()).all()) for t in outs["nccl"])
        results[rank] = (ok["push"], ok["p2p"], diff, finite)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_exchange_modes_agree_across_two_ranks():
    import torch.multiprocessing as mp

    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    ctx = mp.start_processes(_worker, args=(world, _port(), results), nprocs=world, start_method="spawn",
                             join=False)
    for p in ctx.processes:
        p.join(timeout=600)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    for r in range(world):
        push_ok, p2p_ok, diff, finite = results[r]
        print(f"rank {r}: push bit-exact {push_ok}, in place bit-exact {p2p_ok}, max abs difference {diff}")
        assert finite, f"rank {r}: non-finite output"
        assert max(diff.values()) <= 2e-2, f"rank {r}: outputs differ from the NCCL exchange: {diff}"
