"""Per-kernel parity of the CUDA path against the CPU oracle (and torch fp32 references
for the floating-point kernels), called through the C ABI on small seeded inputs."""

import math

import numpy as np
import pytest
import torch

from oracle import recap_oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    from recap_b200 import _lib as lib

    return lib


def _layout(nv, text, text_first, seed=0):
    from recap_b200.sparse.layout import Layout

    perm = np.random.default_rng(seed).permutation(nv)
    return Layout.from_permutation(perm, text_tokens=text, text_first=text_first)


def _strided_qkv(b, h, s, d, seed):
    """bf16 [b, h, s, d] views of [b, s, h, d] storage (the models' layout)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(3):
        x = torch.randn(b, s, h, d, generator=g).to(torch.bfloat16).to(DEV)
        out.append(x.transpose(1, 2))
    return out


def _run_gather(layout, q, k, v, q_mean=True, closure_rank=None):
    from recap_b200.config import OperatorConfig
    from recap_b200.sparse.attention import SparseAttention, SparseGeometry

    geo = SparseGeometry.build(layout, 128)
    cfg = OperatorConfig() if closure_rank is None else OperatorConfig(closure_rank=closure_rank)
    sa = SparseAttention(geo, cfg)
    return sa, sa.prepare(q, k, v, q_mean=q_mean)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nv,text,text_first", [(2048, 0, False), (700, 50, True), (504, 40, False)])
def test_layout_gather_and_pooling(d, nv, text, text_first):
    lay = _layout(nv, text, text_first)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=1)
    _, inp = _run_gather(lay, q, k, v)
    torch.cuda.synchronize()
    sh = inp.shapes
    for src, name in ((q, "q"), (k, "k")):
        ref = lay.reorder(src).reshape(sh.banks, sh.S, d)
        got = getattr(inp, name)
        assert torch.equal(got[:, : sh.S], ref), name
        assert bool((got[:, sh.S:] == 0).all())
    vref = lay.reorder(v).reshape(sh.banks, sh.S, d)
    assert torch.equal(inp.v_t[:, :, : sh.S].transpose(1, 2), vref)
    for src, mean in ((q, inp.q_mean), (k, inp.k_mean), (v, inp.v_mean)):
        ref, _ = orc.pool_blocks(lay.reorder(src).reshape(sh.banks, sh.S, d).float().cpu(), nv)
        assert torch.allclose(mean.cpu(), ref, atol=1e-5, rtol=1e-5)
    kb = inp.k_mean_bf16[:, : sh.nB].float().cpu()
    assert torch.equal(kb, inp.k_mean.cpu().to(torch.bfloat16).float())
    vbt = inp.v_mean_t_bf16[:, :, : sh.nB].transpose(1, 2).float().cpu()
    assert torch.equal(vbt, inp.v_mean.cpu().to(torch.bfloat16).float())


def _selection_matches(got: torch.Tensor, scores: torch.Tensor, keep: int, forced: bool) -> tuple[bool, int]:
    """Selected sets equal to the oracle's, except where a differing block's score ties
    (within 4 fp32 ulp) with the k-th score of its row; the forced partial row/column of
    recap/sparse/attention.py:88-94 must match exactly."""
    ref = orc.topk_mask(scores, keep)
    srt = torch.sort(scores.double(), dim=-1, descending=True).values
    kth = srt[..., keep - 1 : keep]
    tol = 4 * torch.finfo(torch.float32).eps * kth.abs().clamp_min(1e-30)
    tie = (scores.double() - kth).abs() <= tol
    if forced:
        ref[..., -1, :] = True
        ref[..., :, -1] = True
        tie[..., -1, :] = False
        tie[..., :, -1] = False
    diff = got != ref
    return bool((~diff | tie).all()), int(diff.sum())


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nv,keep", [(2048, 4), (700, 2), (118800 // 16, 46), (1400 * 128 - 5, 140)])
def test_pool_select_topk(d, nv, keep):
    from recap_b200 import _lib as lib

    nB = (nv + 127) // 128
    banks = 3
    g = torch.Generator().manual_seed(nv + d)
    qm = torch.randn(banks, nB, d, generator=g).to(DEV)
    km = torch.randn(banks, nB, d, generator=g).to(DEV)
    part = torch.empty(banks, nB, nB, dtype=torch.bool, device=DEV)
    scale = 1 / math.sqrt(d)
    lib.call("recap_pool_select", lib.ptr(qm), lib.ptr(km), banks, nB, d, keep, scale, nv, 128, lib.ptr(part),
             lib.stream_handle(torch.device(DEV)))
    got = part.cpu()
    scores = orc.block_scores(qm.cpu(), km.cpu(), scale)
    ok, n = _selection_matches(got, scores, keep, forced=bool(nv % 128))
    assert ok, f"{n} selections differ beyond fp ties"
    if not nv % 128:
        assert bool((got.sum(-1) == keep).all())


def test_pool_select_ties_take_lower_index():
    from recap_b200 import _lib as lib

    banks, nB, d, keep = 1, 8, 64, 3
    qm = torch.zeros(banks, nB, d)
    qm[..., 0] = 1.0
    km = torch.zeros(banks, nB, d)
    km[0, :, 0] = torch.tensor([0.5, 2.0, 1.0, 1.0, 1.0, 1.0, 0.0, 3.0])
    part = torch.empty(banks, nB, nB, dtype=torch.bool, device=DEV)
    qm_d, km_d = qm.to(DEV), km.to(DEV)
    lib.call("recap_pool_select", lib.ptr(qm_d), lib.ptr(km_d), banks, nB, d, keep, 1.0, nB * 128, 128,
             lib.ptr(part), lib.stream_handle(torch.device(DEV)))
    # scores per row: [0.5, 2, 1, 1, 1, 1, 0, 3] -> top 3 = {7, 1, 2} (block 2 wins the tie)
    assert part[0, 0].cpu().tolist() == [False, True, True, False, False, False, False, True]


def _fmha(q_r, k_r, v_t, part, banks, S, d, nv, all_blocks, out_pos=None, native_out=None, knm=None):
    from recap_b200 import _lib as lib

    out = torch.empty(banks, S, d, dtype=torch.bfloat16, device=DEV) if native_out is None else native_out
    lse = torch.empty(banks, S, dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib.call("recap_block_sparse_fmha", lib.ptr(q_r), lib.ptr(k_r), lib.ptr(v_t), lib.ptr(part), lib.ptr(knm), banks,
             S, d, nv, int(all_blocks), 1 / math.sqrt(d), lib.ptr(out_pos), lib.ptr(out), lib.ptr(lse),
             lib.ptr(status), lib.stream_handle(torch.device(DEV)))
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    return out, lse


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nv,text", [(1024, 0), (700, 50), (300, 9)])
def test_fmha_dense_vs_torch_fp32(d, nv, text):
    lay = _layout(nv, text, True)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=3)
    _, inp = _run_gather(lay, q, k, v, q_mean=False)
    sh = inp.shapes
    out, lse = _fmha(inp.q, inp.k, inp.v_t, None, sh.banks, sh.S, d, nv, True, knm=inp.k_norm_max)
    qr = inp.q[:, : sh.S].float()
    kr = inp.k[:, : sh.S].float()
    vr = inp.v_t[:, :, : sh.S].transpose(1, 2).float()
    s = torch.bmm(qr, kr.transpose(1, 2)) / math.sqrt(d)
    ref_lse = torch.logsumexp(s, -1)
    ref = torch.bmm(torch.softmax(s, -1), vr)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2, f"O max abs err {err}"
    lerr = (lse - ref_lse).abs().max().item()
    assert lerr <= 2e-3, f"LSE max abs err {lerr}"


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nv,text,text_first", [(2048, 0, False), (700, 50, True), (504, 40, False)])
@pytest.mark.parametrize("bound", ["exact", "bounded", "outliers"])
def test_fmha_block_sparse_vs_oracle(d, nv, text, text_first, bound):
    """exact: every block computes its row maximum; bounded: blocks within the |q| |k|
    bound of the running maximum skip it; outliers: a few keys scaled up 60x make the bound
    fail for some warps and blocks, which then fall back to the exact path."""
    lay = _layout(nv, text, text_first)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=4)
    if bound == "outliers":
        g0 = torch.Generator().manual_seed(40)
        idx = torch.randperm(nv + text, generator=g0)[:7]
        k = k.clone()
        k[:, :, idx] *= 60.0
    _, inp = _run_gather(lay, q, k, v, q_mean=False)
    sh = inp.shapes
    g = torch.Generator().manual_seed(5)
    part = torch.rand(sh.banks, sh.nB, sh.nB, generator=g) < 0.3
    if nv % 128:
        part[:, -1, :] = True
        part[:, :, -1] = True
    knm = None if bound == "exact" else inp.k_norm_max
    out, lse = _fmha(inp.q, inp.k, inp.v_t, part.to(DEV), sh.banks, sh.S, d, nv, False, knm=knm)
    kmask = orc.kernel_block_mask(part, sh.S, nv)
    ro, rl = orc.masked_attention(inp.q[:, : sh.S].float().cpu(), inp.k[:, : sh.S].float().cpu(),
                                  inp.v_t[:, :, : sh.S].transpose(1, 2).float().cpu(), kmask, 1 / math.sqrt(d))
    err = (out.float().cpu() - ro).abs().max().item()
    assert err <= 2e-2, f"O max abs err {err}"
    lerr = (lse.cpu() - rl).abs().max().item()
    assert lerr <= 2e-3, f"LSE max abs err {lerr}"


@pytest.mark.parametrize("d", [64, 128])
def test_fmha_uneven_pairs_vs_oracle(d):
    """Query blocks are processed in pairs whose kept lists are split into blocks both keep
    and blocks only one keeps; per-row densities from a single block to every block make
    the two lists of a pair differ in length and run the shared-tile ring through many
    wraps.  An odd block count leaves one CTA with a single query block."""
    nv, text = 128 * 22 + 50, 60
    lay = _layout(nv, text, False)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=14)
    _, inp = _run_gather(lay, q, k, v, q_mean=False)
    sh = inp.shapes
    g = torch.Generator().manual_seed(15)
    dens = torch.rand(sh.banks, sh.nB, 1, generator=g)
    dens[:, ::5] = 0.0  # rows that keep only the forced blocks
    dens[:, 3::7] = 1.0  # rows that keep everything
    part = torch.rand(sh.banks, sh.nB, sh.nB, generator=g) < dens
    part[:, -1, :] = True
    part[:, :, -1] = True
    out, lse = _fmha(inp.q, inp.k, inp.v_t, part.to(DEV), sh.banks, sh.S, d, nv, False, knm=inp.k_norm_max)
    kmask = orc.kernel_block_mask(part, sh.S, nv)
    ro, rl = orc.masked_attention(inp.q[:, : sh.S].float().cpu(), inp.k[:, : sh.S].float().cpu(),
                                  inp.v_t[:, :, : sh.S].transpose(1, 2).float().cpu(), kmask, 1 / math.sqrt(d))
    err = (out.float().cpu() - ro).abs().max().item()
    assert err <= 2e-2, f"O max abs err {err}"
    lerr = (lse.cpu() - rl).abs().max().item()
    assert lerr <= 2e-3, f"LSE max abs err {lerr}"


def _refresh_attention(q_r, k_r, v_t, part, banks, S, d, nv, knm):
    from recap_b200 import _lib as lib

    out = torch.empty(banks, S, d, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(banks, S, dtype=torch.float32, device=DEV)
    head = torch.empty(banks, S, d, dtype=torch.bfloat16, device=DEV)
    head_lse = torch.empty(banks, S, dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib.call("recap_refresh_attention", lib.ptr(q_r), lib.ptr(k_r), lib.ptr(v_t), lib.ptr(part), lib.ptr(knm),
             banks, S, d, nv, 1 / math.sqrt(d), None, lib.ptr(out), lib.ptr(lse), lib.ptr(head),
             lib.ptr(head_lse), lib.ptr(status), lib.stream_handle(torch.device(DEV)))
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    return out, lse, head, head_lse


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nv,text,text_first,dens", [(2048, 0, False, "flat"), (700, 50, True, "flat"),
                                                     (504, 40, False, "flat"), (128 * 22 + 50, 60, False, "uneven"),
                                                     (128 * 21, 0, False, "uneven")])
def test_refresh_attention_head_and_dense(d, nv, text, text_first, dens):
    """The fused REFRESH pass: its head output and LSE equal the block-sparse pass's bit for
    bit on the sparse query blocks (same kept blocks in the same order, same arithmetic) and
    within tolerance on the dense ones (every key block, in the order their pairing gives),
    and its dense output and LSE
    match exact fp32 attention within the parity tolerance (max-abs 2e-2 on O, 2e-3 on LSE).
    Uneven densities (rows keeping one block next to rows keeping all) give pairs whose kept
    lists differ in length, so the middle rounds load separate tiles while the first and
    last rounds share them; an odd block count leaves one CTA with a single query block."""
    lay = _layout(nv, text, text_first)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=21)
    _, inp = _run_gather(lay, q, k, v, q_mean=False)
    sh = inp.shapes
    g = torch.Generator().manual_seed(22)
    if dens == "flat":
        part = torch.rand(sh.banks, sh.nB, sh.nB, generator=g) < 0.3
    else:
        rate = torch.rand(sh.banks, sh.nB, 1, generator=g)
        rate[:, ::5] = 0.0
        rate[:, 3::7] = 1.0
        part = torch.rand(sh.banks, sh.nB, sh.nB, generator=g) < rate
    # every row keeps at least one block, as the top-k selection guarantees (keep >= 1)
    part |= torch.eye(sh.nB, dtype=torch.bool)
    if nv % 128:
        part[:, -1, :] = True
        part[:, :, -1] = True
    part = part.to(DEV)
    out, lse, head, head_lse = _refresh_attention(inp.q, inp.k, inp.v_t, part, sh.banks, sh.S, d, nv,
                                                  inp.k_norm_max)
    ref_head, ref_head_lse = _fmha(inp.q, inp.k, inp.v_t, part, sh.banks, sh.S, d, nv, False, knm=inp.k_norm_max)
    # query blocks below dense_start (every row the refinement reads): the same bits; the
    # dense query blocks attend every key block, in an order that depends on their pairing
    ds = sh.nB - 1 if (nv % 128 and sh.S > nv) else sh.nB
    assert torch.equal(head[:, : ds * 128], ref_head[:, : ds * 128])
    assert torch.equal(head_lse[:, : ds * 128], ref_head_lse[:, : ds * 128])
    if ds * 128 < sh.S:
        assert (head[:, ds * 128:].float() - ref_head[:, ds * 128:].float()).abs().max().item() <= 2e-2
        assert (head_lse[:, ds * 128:] - ref_head_lse[:, ds * 128:]).abs().max().item() <= 2e-3
    qr = inp.q[:, : sh.S].float()
    kr = inp.k[:, : sh.S].float()
    vr = inp.v_t[:, :, : sh.S].transpose(1, 2).float()
    s = torch.bmm(qr, kr.transpose(1, 2)) / math.sqrt(d)
    ref_lse = torch.logsumexp(s, -1)
    ref = torch.bmm(torch.softmax(s, -1), vr)
    err = (out.float() - ref).abs().max().item()
    lerr = (lse - ref_lse).abs().max().item()
    print(f"dense O max abs {err:.3e}, LSE max abs {lerr:.3e}")
    assert err <= 2e-2, f"O max abs err {err}"
    assert lerr <= 2e-3, f"LSE max abs err {lerr}"


def test_layout_key_norm_bounds():
    """The layout pass's norm bounds: the largest |k| over each 128-token block (text
    included) and |bf16(kbar)| of each video block."""
    nv, text, d = 700, 50, 128
    lay = _layout(nv, text, True)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=41)
    _, inp = _run_gather(lay, q, k, v, q_mean=False)
    torch.cuda.synchronize()
    sh = inp.shapes
    kr = inp.k.float().cpu()  # [banks, S_pad, d], zero past S
    ref = kr.norm(dim=-1).reshape(sh.banks, -1, 128).amax(-1)
    assert torch.allclose(inp.k_norm_max.cpu(), ref, rtol=1e-5, atol=1e-5)
    kb = inp.k_mean.cpu().to(torch.bfloat16).float().norm(dim=-1)
    assert torch.allclose(inp.k_mean_norm.cpu(), kb, rtol=1e-5, atol=1e-5)


def test_exp2_poly_vs_exp2f():
    """The softmax's FP32-pipe exponential against exp2 in double precision on the GPU:
    relative error below 1e-4 over the range it is used on, and a non-negative value below
    2^-124 under it (where it stands for zero)."""
    lib = _lib()
    y = torch.cat([torch.linspace(-125.0, 127.0, 200001), torch.linspace(-8.0, 8.0, 100001),
                   torch.tensor([0.0, -0.5, 0.5, -1e-7, 1e-7, -124.999, 126.9])]).to(DEV)
    out = torch.empty_like(y)
    lib.call("recap_exp2_check", lib.ptr(y), lib.ptr(out), y.numel(), lib.stream_handle(torch.device(DEV)))
    ref = torch.exp2(y.double())
    rel = ((out.double() - ref).abs() / ref).max().item()
    assert rel <= 1e-4, rel
    low = torch.tensor([-126.0, -200.0, -1e30, float("-inf")], device=DEV)
    out_low = torch.empty_like(low)
    lib.call("recap_exp2_check", lib.ptr(low), lib.ptr(out_low), low.numel(), lib.stream_handle(torch.device(DEV)))
    torch.cuda.synchronize()
    assert bool((out_low >= 0).all()) and float(out_low.max()) <= 2.0 ** -124


def test_bounded_wait_runs_out_without_fault():
    """The bounded mbarrier wait of every kernel, driven to its limit on purpose: a
    barrier nothing arrives on.  The waiter records the timeout in the status word and
    raises the block's abort flag; the second waiter leaves through the flag long before
    its own (4x) limit; the context stays usable and the operator's status check raises."""
    from recap_b200 import Operator, OperatorConfig, _lib as lib
    from recap_b200.sparse import Layout, SparseGeometry

    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    result = torch.full((3,), -1, dtype=torch.int64, device=DEV)
    limit_ns = 50_000_000
    lib.call("recap_wait_selftest", lib.ptr(status), limit_ns, lib.ptr(result), lib.stream_handle(torch.device(DEV)))
    torch.cuda.synchronize()
    assert int(status.item()) == 106
    r = result.cpu().tolist()
    assert r[0] == 0 and r[1] == 0, r
    assert limit_ns * 0.9 <= r[2] < 3 * limit_ns, r
    # the context is still usable
    x = torch.arange(1000, device=DEV, dtype=torch.float32)
    assert float(x.sum()) == 499500.0
    # the operator's status check reports a set status word, then clears it
    lay = Layout.from_permutation(np.arange(1024), text_tokens=0, text_first=False)
    op = Operator.build(OperatorConfig(), SparseGeometry.build(lay, 128), n_layers=1)
    word = op.status_word(torch.device(DEV))
    lib.call("recap_wait_selftest", lib.ptr(word), limit_ns, lib.ptr(result), lib.stream_handle(torch.device(DEV)))
    with pytest.raises(RuntimeError, match="device timeout"):
        op.check_device_status()
    op.check_device_status()  # cleared


def test_fmha_native_output_positions():
    nv, text, d = 700, 50, 64
    lay = _layout(nv, text, True)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=6)
    _, inp = _run_gather(lay, q, k, v, q_mean=False)
    sh = inp.shapes
    out_r, lse_r = _fmha(inp.q, inp.k, inp.v_t, None, sh.banks, sh.S, d, nv, True)
    out_n, lse_n = _fmha(inp.q, inp.k, inp.v_t, None, sh.banks, sh.S, d, nv, True,
                         out_pos=lay.gather_rows(torch.device(DEV)))
    fwd = lay.gather_rows(torch.device(DEV)).long()
    assert torch.equal(out_n[:, fwd], out_r)
    assert torch.equal(lse_n[:, fwd], lse_r)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nv,text,text_first", [(2048, 0, False), (700, 50, True)])
def test_closure_statistics_vs_oracle(d, nv, text, text_first):
    from recap_b200 import _lib as lib

    lay = _layout(nv, text, text_first)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=7)
    sa, inp = _run_gather(lay, q, k, v, q_mean=False)
    sh = inp.shapes
    ctx = sa.coarse_tail_context(inp, 1 / math.sqrt(d))
    torch.cuda.synchronize()
    k_r = inp.k[:, : sh.S].float().cpu()
    v_r = inp.v_t[:, :, : sh.S].transpose(1, 2).float().cpu()
    km, counts = orc.pool_blocks(k_r, nv)
    # centred keys written by the layout pass (bf16, transposed, zero outside video)
    blk = torch.arange(nv) // 128
    kc_ref = (k_r[:, :nv] - km[:, blk]).transpose(1, 2)
    kct = inp.k_centred_t.float().cpu()
    assert torch.allclose(kct[:, :, :nv], kc_ref.to(torch.bfloat16).float(), atol=1e-2, rtol=1e-2)
    assert bool((kct[:, :, nv:] == 0).all())
    # C_vk on tensor cores from bf16-rounded centred keys
    cvk = orc.cross_covariance(k_r, v_r, km, counts, nv)
    err = (ctx["cvk"].cpu() - cvk).abs().max().item()
    assert err <= 2e-3 * max(1.0, float(cvk.abs().max())), err
    basis = ctx["basis"].cpu()
    var = orc.fold_rank(orc.rotated_variance(k_r, basis, nv), 4)
    assert torch.allclose(ctx["variance"].cpu(), var, atol=1e-4, rtol=1e-3), (ctx["variance"].cpu() - var).abs().max()
    # the basis is an ordered eigenbasis of the pooled within-block scatter
    scat = orc.within_block_scatter(k_r, km, counts, nv)
    evals = torch.linalg.eigvalsh(scat.double())
    proj = torch.einsum("bdi,bde,bei->bi", basis.double(), scat.double(), basis.double())
    assert torch.allclose(torch.sort(proj, -1).values, evals, atol=1e-3, rtol=1e-3)
    eye = torch.eye(d, dtype=torch.float64).expand(sh.banks, d, d)
    assert torch.allclose(basis.double().transpose(1, 2) @ basis.double(), eye, atol=1e-4)
    pooled = (orc.rotated_variance(k_r, basis, nv) * counts.view(1, -1, 1)).sum(1)
    assert bool((pooled[:, :-1] >= pooled[:, 1:] - 1e-4 * pooled.abs().max()).all()), "basis not ordered"
    assert torch.equal(ctx["basis_t"].float().cpu(), basis.transpose(1, 2).to(torch.bfloat16).float())
    # second call: the basis is known, the layout pass folds the variances itself
    inp2 = sa.prepare(q, k, v, q_mean=False)
    assert inp2.variance is not None
    ctx2 = sa.coarse_tail_context(inp2, 1 / math.sqrt(d))
    torch.cuda.synchronize()
    assert torch.allclose(ctx2["variance"].cpu(), var, atol=1e-4, rtol=2e-3), (ctx2["variance"].cpu() - var).abs().max()
    assert torch.equal(ctx2["variance_bf16"][:, : sh.nB].float().cpu(), ctx2["variance"].cpu().to(torch.bfloat16).float())
    del lib


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("rank", [1, 3, 8, 20])
def test_gather_folded_variance_ranks(d, rank):
    """The layout pass's rank-folded variances (second call, basis known) at every rank
    its tensor-core rotation takes (1 .. 8, zero columns past the rank) and one above,
    which goes to the per-column kernel; a partial last video block (700 tokens)."""
    nv, text = 700, 50
    lay = _layout(nv, text, True)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=11)
    sa, inp = _run_gather(lay, q, k, v, q_mean=False, closure_rank=rank)
    ctx = sa.coarse_tail_context(inp, 1 / math.sqrt(d))
    inp2 = sa.prepare(q, k, v, q_mean=False)
    ctx2 = sa.coarse_tail_context(inp2, 1 / math.sqrt(d))
    torch.cuda.synchronize()
    from recap_b200 import _lib as lib

    assert (inp2.variance is not None) == (rank <= lib.load().recap_gather_max_rank())
    k_r = inp.k[:, : inp.shapes.S].float().cpu()
    var = orc.fold_rank(orc.rotated_variance(k_r, ctx["basis"].cpu(), nv), rank)
    got = ctx2["variance"].cpu()
    assert torch.allclose(got, var, atol=1e-5, rtol=2e-5), (got - var).abs().max()


@pytest.mark.parametrize("d", [64, 128])
def test_gather_folded_variance_large_block_means(d):
    """Keys whose block means are large against their within-block spread (smooth fields
    plus noise, as the video models produce).  The leading columns rotate the raw keys on
    the tensor cores; their fp32 accumulation loses ~2^-23 |mean| / |spread| of the
    spread, as the reference's own tensor-core rotation of the raw keys does
    (recap/kernels/closure_stats.py:96-189), and the folded tail columns, which come from
    the trace identity sum_c var(K U[:, c]) = trace(cov K) (exact for the orthonormalized
    basis), inherit that through the leading variances: within 2e-4 of the fp64 oracle on
    this data, against 7e-5 that a basis orthonormal only to eigh's ~3e-5 added alone."""
    nv, text = 128 * 20 + 37, 30
    lay = _layout(nv, text, False, seed=3)
    g = torch.Generator().manual_seed(21)
    tok = torch.arange(nv + text, dtype=torch.float32)
    field = 6.0 * torch.cos(tok[:, None] * 0.002 + torch.rand(d, generator=g)[None, :] * 6.28)
    ks = []
    for _ in range(3):
        x = field + 0.5 * torch.randn(nv + text, d, generator=g)
        ks.append(x.reshape(1, 1, nv + text, d).to(torch.bfloat16).to(DEV))
    q, k, v = ks
    sa, inp = _run_gather(lay, q, k, v, q_mean=False, closure_rank=4)
    ctx = sa.coarse_tail_context(inp, 1 / math.sqrt(d))
    inp2 = sa.prepare(q, k, v, q_mean=False)
    assert inp2.variance is not None
    torch.cuda.synchronize()
    k_r = inp.k[:, : inp.shapes.S].float().cpu()
    var = orc.fold_rank(orc.rotated_variance(k_r, ctx["basis"].cpu(), nv), 4)
    got = inp2.variance.cpu()
    rel = ((got - var).abs() / var.abs().clamp_min(1e-6))
    assert float(rel.max()) <= 2e-4, float(rel.max())


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("nv,text,text_first", [(2048, 0, False), (700, 50, True)])
def test_coarse_tail_vs_oracle(d, nv, text, text_first):
    _check_coarse_tail(d, nv, text, text_first, None)


@pytest.mark.parametrize("mode", ["exact", "bounded", "outliers"])
def test_coarse_tail_bound_paths_vs_oracle(mode):
    """exact: every tile computes its maximum and exchanges it between the two threads of
    a row (the operator's default); bounded: tiles within the |q| |kbar| logit bound skip
    it; outliers: a few keys scaled up 60x make the bound fail for some warps and tiles,
    which then mix exact and bounded tiles."""
    _check_coarse_tail(128, 128 * 290 + 77, 50, True, None, mode=mode)


@pytest.mark.parametrize("d,rank", [(128, 0), (64, 0), (128, 20), (64, 60), (64, 62), (128, 1)])
def test_coarse_tail_ranks_vs_oracle(d, rank):
    """The quadratic term over a folded variance (rank + 4 columns, one to four K-steps;
    rank 62 of 64 is past the fold and runs unfolded) and over the full head dimension
    (rank 0: not folded), with 291 key blocks: three tiles of block means through the
    operand rings, the last one mostly padding."""
    _check_coarse_tail(d, 128 * 290 + 77, 50, True, rank)


def _check_coarse_tail(d, nv, text, text_first, rank, mode="exact"):
    lay = _layout(nv, text, text_first)
    q, k, v = _strided_qkv(1, 2, nv + text, d, seed=8)
    if mode == "outliers":
        g0 = torch.Generator().manual_seed(42)
        idx = torch.randperm(nv, generator=g0)[:2000]
        k = k.clone()
        k[:, :, idx] *= 60.0
    sa, inp = _run_gather(lay, q, k, v, q_mean=True, closure_rank=rank)
    sh = inp.shapes
    scale = 1 / math.sqrt(d)
    part = sa.head_partition(inp, scale)
    ctx = sa.coarse_tail_context(inp, scale)
    old = torch.randn(sh.banks, sh.rows, generator=torch.Generator().manual_seed(9)).to(DEV)
    out, lse, center = sa.coarse_tail_apply(inp, ctx, part.reshape(sh.banks, sh.nB, sh.nB), scale, old_lse=old,
                                            logit_bound=mode != "exact")
    torch.cuda.synchronize()
    q_r = inp.q[:, : sh.S].float().cpu()
    k_r = inp.k[:, : sh.S].float().cpu()
    v_r = inp.v_t[:, :, : sh.S].transpose(1, 2).float().cpu()
    km, counts = orc.pool_blocks(k_r, nv)
    vm, _ = orc.pool_blocks(v_r, nv)
    basis = ctx["basis"].cpu()
    var = ctx["variance"].cpu()
    qsq = orc.rotated_query_square(q_r[:, :nv], basis, torch.bfloat16)
    drift = orc.value_drift(q_r[:, :nv], ctx["cvk"].cpu(), scale, torch.bfloat16)
    ro, rl = orc.coarse_tail(q_r, km, vm, var, counts, part.reshape(sh.banks, sh.nB, sh.nB).cpu(), qsq, drift,
                             scale, 2.0, sh.rows, torch.bfloat16)
    err = (out.float().cpu() - ro).abs().max().item()
    assert err <= 2e-2, f"coarse O max abs err {err}"
    fin = torch.isfinite(rl)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    lerr = (lse.cpu()[fin] - rl[fin]).abs().max().item()
    assert lerr <= 2e-3, f"coarse LSE err {lerr}"
    rc = orc.drift_center(rl, old.cpu())
    assert torch.allclose(center.cpu(), rc, atol=1e-3)


def test_refresh_detail_vs_oracle():
    from recap_b200 import _lib as lib

    banks, nv, text, d = 2, 700, 50, 64
    S = nv + text
    rows = (nv // 128) * 128
    g = torch.Generator().manual_seed(10)
    perm = torch.randperm(nv, generator=g)
    full_o = torch.randn(banks, S, d, generator=g).to(torch.bfloat16)
    full_lse = torch.randn(banks, S, generator=g) + 4
    head_o = torch.randn(banks, S, d, generator=g).to(torch.bfloat16)
    head_lse = full_lse[:, (text + perm).tolist() + list(range(text))] - torch.rand(banks, S, generator=g) * 2
    go = torch.randn(banks, rows, d, generator=g).to(torch.bfloat16)
    gl = torch.randn(banks, rows, generator=g) + 2
    det0 = (torch.randn(banks, rows, d, generator=g) * 0.1).half()
    dl0 = torch.randn(banks, rows, generator=g) * 0.1
    old = gl + torch.randn(banks, rows, generator=g) * 0.1
    center = (gl - old).mean(1)
    det = det0.clone().to(DEV)
    dl = dl0.clone().to(DEV)
    n = lib.load().recap_refresh_partials(banks, nv)
    partials = torch.empty(n, 2, device=DEV)
    stats = torch.zeros(2, device=DEV)
    # keep every device buffer referenced until the kernel has run (a temporary freed
    # while its pointer is in flight would be reused by the caching allocator)
    dev = {name: t.contiguous().to(DEV) for name, t in dict(
        full_o=full_o, full_lse=full_lse, head_o=head_o, head_lse=head_lse, go=go, gl=gl, old=old, center=center,
        perm=perm.to(torch.int32)).items()}
    lib.call("recap_refresh_detail", lib.ptr(dev["full_o"]), lib.ptr(dev["full_lse"]), lib.ptr(dev["head_o"]),
             lib.ptr(dev["head_lse"]), lib.ptr(dev["go"]), lib.ptr(dev["gl"]), lib.ptr(dev["perm"]), banks, S,
             d, nv, text, lib.ptr(det), lib.ptr(dl), 1, lib.ptr(dev["old"]), lib.ptr(dev["center"]), lib.ptr(partials),
             lib.ptr(stats), lib.stream_handle(torch.device(DEV)))
    torch.cuda.synchronize()
    rdet, rdl, rstats = orc.refresh_detail(full_o.float(), full_lse, head_o.float(), head_lse, go.float(), gl,
                                           perm.numpy(), text, det0.float(), dl0, old, center)
    assert (det.float().cpu() - rdet.float()).abs().max() <= 2e-3 * max(1.0, float(rdet.float().abs().max()))
    assert torch.allclose(dl.cpu(), rdl, atol=1e-4)
    assert torch.allclose(stats.cpu(), rstats.float(), rtol=1e-4)
