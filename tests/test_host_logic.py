"""Host-side logic that needs no GPU: config, layout, geometry, the C ABI's exports."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import recap_oracle as orc
from recap_b200 import OperatorConfig, keep_blocks
from recap_b200.sparse.attention import Shapes, SparseGeometry
from recap_b200.sparse.layout import Layout

REPO = Path(__file__).resolve().parents[1]


def test_config_validation_matches_reference_rules():
    OperatorConfig().validate()
    for bad in [dict(head_density=0.0), dict(head_density=1.0), dict(closure_gate_theta=0.0),
                dict(closure_rank=-1), dict(rerank_min_overlap=1.5), dict(bank_chunks=0), dict(block_size=64)]:
        with pytest.raises(ValueError):
            OperatorConfig(**bad).validate()


def test_keep_blocks_matches_oracle():
    for density in (0.1, 0.15, 0.2, 0.25, 0.34, 0.5):
        for nb in (1, 3, 16, 256, 351, 929):
            assert keep_blocks(density, nb) == orc.keep_blocks(density, nb)


@pytest.mark.parametrize("text_first", [False, True])
def test_layout_gather_rows_roundtrip(text_first):
    perm = np.random.default_rng(0).permutation(300)
    lay = Layout.from_permutation(perm, text_tokens=37, text_first=text_first)
    x = torch.randn(2, 3, 337, 8)
    assert torch.equal(lay.restore(lay.reorder(x)), x)
    rows = lay.gather_rows(torch.device("cpu")).long()
    assert torch.equal(x[..., rows, :], lay.reorder(x))
    fwd, inv = orc.gather_indices(torch.as_tensor(perm), 37, text_first)
    assert torch.equal(rows, fwd)
    # restore writes reordered row r to native row rows[r]
    y = torch.empty_like(x)
    y[..., rows, :] = lay.reorder(x)
    assert torch.equal(y, x)


def test_layout_rejects_bad_permutation():
    with pytest.raises(ValueError):
        Layout.from_permutation(np.array([0, 0, 1]), text_tokens=0, text_first=False)


@pytest.mark.parametrize("nv,text,expect", [
    (118800, 256, dict(NB=931, nB=929, rows=118784, dense_start=928)),
    (32760, 0, dict(NB=256, nB=256, rows=32640, dense_start=256)),
    (44880, 226, dict(NB=353, nB=351, rows=44800, dense_start=350)),
    (2048, 0, dict(NB=16, nB=16, rows=2048, dense_start=16)),
])
def test_shapes_of_benchmark_configs(nv, text, expect):
    q = torch.empty(1, 2, nv + text, 64, device="meta")
    sh = Shapes.of(q, nv)
    for k, v in expect.items():
        assert getattr(sh, k) == v


def test_geometry_block_counts():
    lay = Layout.from_permutation(np.arange(300), text_tokens=0, text_first=False)
    g = SparseGeometry.build(lay, 128)
    assert g.n_blocks == 3 and g.block_counts.tolist() == [128.0, 128.0, 44.0]
    with pytest.raises(ValueError):
        SparseGeometry.build(lay, 64)


def _declared_symbols():
    text = (REPO / "include" / "recap_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t)\s+(recap_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from recap_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    declared = _declared_symbols()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures must cover the header"
    assert _lib.load().recap_abi_version() == _lib.ABI_VERSION


def test_library_rejects_bad_shapes_without_a_gpu():
    from recap_b200 import _lib

    lib = _lib.load()
    # D must be 64 or 128: rejected on the host before any device call
    assert lib.recap_pool_select(None, None, 1, 4, 96, 1, 1.0, 512, 128, None, None) == _lib.RECAP_ERR_SHAPE
    # more key blocks than the attention kernels take (2048)
    assert lib.recap_pool_select(None, None, 1, 2049, 128, 1, 1.0, 2049 * 128, 128, None, None) == \
        _lib.RECAP_ERR_SHAPE
    assert lib.recap_closure_workspace_floats(2, 64, 2048) == 2 * 2 * 1 * 64 * 64


def test_bench_clock_summary_merges_nvml_polls_and_reasons(tmp_path):
    """The bench's clock record: nvidia-smi rows after the start mark plus NVML polls,
    median SM clock, the largest max clock, and the throttle reasons either source saw."""
    import sys

    sys.path.insert(0, str(REPO))
    import bench

    c = bench.ClockSampler("00000000:00:00.0")
    c.path = tmp_path / "clocks.csv"
    c.path.write_text("0, 1965, 1965, 300, 0x0, Not Active, Not Active, Not Active, Not Active\n"
                      "0, 1800, 1965, 900, 0x4, Not Active, Not Active, Not Active, Active\n")
    c.skip = 1  # the first row was taken before the timed region
    c.polled = [(1700.0, 1965.0, 0x4), (1900.0, 1965.0, 0x0), (1850.0, 1965.0, 0x20)]
    s = c.summary()
    assert s["samples"] == 4
    assert s["sm_mhz"] == 1850.0  # sorted 1700, 1800, 1850, 1900 -> element 2
    assert s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    c.path = tmp_path / "missing.csv"
    c.polled = []
    assert c.summary()["samples"] == 0


def test_bench_kept_tile_flops_counts_real_tokens():
    """4 m n d per kept 128x128 tile, with the partial last block's real token count and the
    shared text row and column always counted."""
    import sys

    sys.path.insert(0, str(REPO))
    import bench

    nv, S, d = 300, 310, 64  # blocks of 128, 128, 44 video tokens + 10 text: NB = 3, shared last block
    part = torch.zeros(1, 1, 3, 3, dtype=torch.bool)
    part[0, 0, 0, 1] = True
    counts = [128.0, 128.0, 54.0]
    want = 4 * d * (counts[0] * counts[1] + sum(counts[i] * counts[2] for i in range(2)) +
                    sum(counts[2] * counts[j] for j in range(3)))
    assert bench.kept_tile_flops(part, S, nv, d) == pytest.approx(want)
