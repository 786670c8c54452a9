"""The sequence-parallel attention path on one GPU: the ranks' token shards emulated as
separate buffers on the device (the kernels take any reachable address, local or a peer's
over NVLink).  ``Operator.attend_sharded`` must give bit for bit what ``Operator.attend``
gives on the gathered heads, through REFRESH -> SPARSE -> revalidating REFRESH -> SPARSE,
with the layout pass reading each rank's projection shard and the SPARSE epilogue storing
each row into the shard of the rank that owns the token."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _shards(full: torch.Tensor, world: int):
    """[S, ...] -> per-rank contiguous buffers of S / world tokens."""
    s = full.shape[0] // world
    return [full[q * s:(q + 1) * s].contiguous() for q in range(world)]


@pytest.mark.parametrize("mode", ["in_place", "push"])
@pytest.mark.parametrize("world,rank,text,text_first,d", [(2, 0, 64, False, 128), (2, 1, 64, False, 128),
                                                          (4, 2, 0, False, 64), (4, 3, 96, True, 128)])
def test_sharded_attention_matches_plain(world, rank, text, text_first, d, mode):
    """``in_place``: the layout pass reads every rank's projection shard; ``push``: every
    rank first writes its rows of this rank's heads into this rank's receive buffer
    (``ShardedIO.push``, copy-engine copies) and the layout pass reads that locally."""
    from recap_b200 import REFRESH, SPARSE, Operator, OperatorConfig
    from recap_b200.sparse import Layout, SparseGeometry
    from recap_b200.ulysses import ShardedIO

    H = 2 * world
    nv = 128 * 20 - 16 * world  # a partial video block; S divisible by the rank count
    S = nv + text
    assert S % world == 0
    perm = np.random.default_rng(3).permutation(nv)
    layout = Layout.from_permutation(perm, text_tokens=text, text_first=text_first)
    geo = SparseGeometry.build(layout, 128)
    cfg = OperatorConfig(head_density=0.25)
    plain = Operator.build(cfg, geo, n_layers=1)
    sharded = Operator.build(cfg, geo, n_layers=1)
    g = torch.Generator().manual_seed(7)
    s = S // world
    h = H // world
    head0 = rank * h
    out_bufs = [torch.zeros(s, H, d, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    recv_bufs = [torch.zeros(S, 3, h, d, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    steps = [(0, REFRESH), (1, SPARSE), (2, REFRESH), (3, SPARSE)]
    base = torch.randn(S, 3, H, d, generator=g)
    for step, kind in steps:
        full = (base + 0.05 * step * torch.randn(S, 3, H, d, generator=g)).to(torch.bfloat16).to(DEV)
        qkv_bufs = _shards(full, world)
        nbytes = [t.numel() * 2 for t in qkv_bufs]
        qkv = SimpleNamespace(ptrs=[t.data_ptr() for t in qkv_bufs], world=world, rank=rank,
                              device=torch.device(DEV), nbytes=min(nbytes))
        outp = SimpleNamespace(ptrs=[t.data_ptr() for t in out_bufs], world=world, rank=rank,
                               device=torch.device(DEV), nbytes=out_bufs[0].numel() * 2)
        if mode == "push":
            recv = SimpleNamespace(ptrs=[t.data_ptr() for t in recv_bufs], world=world, rank=rank,
                                   device=torch.device(DEV), nbytes=recv_bufs[0].numel() * 2)
            for src in range(world):  # every rank pushes its shard (emulated one after another)
                src_out = SimpleNamespace(**{**vars(outp), "rank": src})
                src_recv = SimpleNamespace(**{**vars(recv), "rank": src})
                ShardedIO(None, src_out, total_heads=H, dim=d, seq=S, recv=src_recv).push(qkv_bufs[src])
            io = ShardedIO(None, outp, total_heads=H, dim=d, seq=S, recv=recv)
        else:
            io = ShardedIO(qkv, outp, total_heads=H, dim=d, seq=S)
        assert io.head0 == head0 and io.heads == h
        q, k, v = (full[:, i, head0:head0 + h].permute(1, 0, 2).unsqueeze(0) for i in range(3))
        plain.begin_step(step, kind)
        ref = plain.attend(0, q, k, v)
        sharded.begin_step(step, kind)
        for b in out_bufs:
            b.zero_()
        sharded.attend_sharded(0, io)
        torch.cuda.synchronize()
        got = torch.cat([b[:, head0:head0 + h] for b in out_bufs]).permute(1, 0, 2).unsqueeze(0)
        assert torch.equal(got, ref), f"step {step} ({kind}): max diff {(got.float() - ref.float()).abs().max()}"
        # the other heads' columns of every shard are left alone
        others = [torch.cat([b[:, :head0], b[:, head0 + h:]], 1) for b in out_bufs]
        assert all(bool((o == 0).all()) for o in others)
        assert torch.equal(plain.banks[0][0].partition, sharded.banks[0][0].partition)
    plain.check_device_status()
    sharded.check_device_status()
