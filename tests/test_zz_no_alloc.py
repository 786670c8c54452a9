"""recap_refresh_detail_noalloc: the refinement write for callers that may not allocate
device memory (hosts that hand a plugin only buffers they planned themselves, or step
loops that cannot afford cudaMalloc's device synchronisation).  It keeps its validation
scratch in an array inside the library instead of taking a caller buffer.

Checked through the C ABI against recap_refresh_detail (caller scratch) on the same
inputs, on two calls in a row, so that the second call also shows that whatever the
first left in the shared array does not leak into the result.  This file is collected
last so that a failure here stops a -x run only after every other test has run."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(seed: int, banks: int, nv: int, text: int, d: int):
    S = nv + text
    rows = (nv // 128) * 128
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(nv, generator=g)
    full_o = torch.randn(banks, S, d, generator=g).to(torch.bfloat16)
    full_lse = torch.randn(banks, S, generator=g) + 4
    head_o = torch.randn(banks, S, d, generator=g).to(torch.bfloat16)
    head_lse = full_lse[:, (text + perm).tolist() + list(range(text))] - torch.rand(banks, S, generator=g) * 2
    go = torch.randn(banks, rows, d, generator=g).to(torch.bfloat16)
    gl = torch.randn(banks, rows, generator=g) + 2
    det = (torch.randn(banks, rows, d, generator=g) * 0.1).half()
    dl = torch.randn(banks, rows, generator=g) * 0.1
    old = gl + torch.randn(banks, rows, generator=g) * 0.1
    center = (gl - old).mean(1)
    t = dict(full_o=full_o, full_lse=full_lse, head_o=head_o, head_lse=head_lse, go=go, gl=gl, old=old,
             center=center, perm=perm.to(torch.int32), det=det, dl=dl)
    return {k: v.contiguous().to(DEV) for k, v in t.items()}


def _run(lib, name: str, x: dict, banks: int, nv: int, text: int, d: int):
    det = x["det"].clone()
    dl = x["dl"].clone()
    stats = torch.full((2,), float("nan"), device=DEV)
    head = [lib.ptr(x["full_o"]), lib.ptr(x["full_lse"]), lib.ptr(x["head_o"]), lib.ptr(x["head_lse"]),
            lib.ptr(x["go"]), lib.ptr(x["gl"]), lib.ptr(x["perm"]), banks, nv + text, d, nv, text, lib.ptr(det),
            lib.ptr(dl), 1, lib.ptr(x["old"]), lib.ptr(x["center"])]
    stream = lib.stream_handle(torch.device(DEV))
    if name == "recap_refresh_detail":
        n = lib.load().recap_refresh_partials(banks, nv)
        partials = torch.empty(max(n, 1), 2, device=DEV)
        lib.call(name, *head, lib.ptr(partials), lib.ptr(stats), stream)
    else:
        lib.call(name, *head, lib.ptr(stats), stream)
    torch.cuda.synchronize()
    return det, dl, stats


@pytest.mark.parametrize("d", [64, 128])
def test_noalloc_refresh_matches_caller_scratch_twice(d):
    from recap_b200 import _lib as lib

    banks, nv, text = 3, 1300, 40
    for call, seed in enumerate((11, 12)):
        x = _inputs(seed + d, banks, nv, text, d)
        det_a, dl_a, st_a = _run(lib, "recap_refresh_detail", x, banks, nv, text, d)
        det_b, dl_b, st_b = _run(lib, "recap_refresh_detail_noalloc", x, banks, nv, text, d)
        assert torch.equal(det_a, det_b), f"call {call}: refinement value differs"
        assert torch.equal(dl_a, dl_b), f"call {call}: refinement log-mass differs"
        assert bool(torch.isfinite(st_b).all()), f"call {call}: stats not written"
        assert torch.allclose(st_a, st_b, rtol=1e-6, atol=0.0), (call, st_a.tolist(), st_b.tolist())


def test_noalloc_refresh_rejects_sizes_beyond_its_array():
    """One bank past the limit is refused before any device work, with its own error.
    The buffers are real and correctly sized, so the call would stay in bounds even if the
    host check were missing."""
    from recap_b200 import _lib as lib

    lib_ = lib.load()
    banks, nv, d = 65, 65536, 64  # 65 * 65536 / 32 = 133120 > 131072 chunks
    assert lib_.recap_refresh_partials(64, nv) == 131072
    rows = nv
    bf = dict(dtype=torch.bfloat16, device=DEV)
    f32 = dict(dtype=torch.float32, device=DEV)
    full_o = torch.zeros(banks, nv, d, **bf)
    head_o = torch.zeros(banks, nv, d, **bf)
    go = torch.zeros(banks, rows, d, **bf)
    det = torch.zeros(banks, rows, d, dtype=torch.float16, device=DEV)
    lse = torch.zeros(banks, nv, **f32)
    gl = torch.zeros(banks, rows, **f32)
    dl = torch.zeros(banks, rows, **f32)
    old = torch.zeros(banks, rows, **f32)
    center = torch.zeros(banks, **f32)
    perm = torch.arange(nv, dtype=torch.int32, device=DEV)
    stats = torch.zeros(2, **f32)
    args = [lib.ptr(full_o), lib.ptr(lse), lib.ptr(head_o), lib.ptr(lse), lib.ptr(go), lib.ptr(gl), lib.ptr(perm),
            banks, nv, d, nv, 0, lib.ptr(det), lib.ptr(dl), 1, lib.ptr(old), lib.ptr(center), lib.ptr(stats),
            lib.stream_handle(torch.device(DEV))]
    assert lib_.recap_refresh_detail_noalloc(*args) == lib.RECAP_ERR_SCRATCH_LIMIT
    with pytest.raises(ValueError, match="fixed array"):
        lib.call("recap_refresh_detail_noalloc", *args)
    torch.cuda.synchronize()
