"""Benchmark: RECAP's corrected sparse attention operator on B200.

Workload: one HunyuanVideo-shaped 720p 129-frame attention layer,
24 heads x 128, 118800 video tokens (33x45x80 Hilbert-ordered) + 256 text tokens
(text last), keep ratio 0.1 (93 of 929 key blocks), refinement bank of all heads in HBM.
A step is one corrected SPARSE layer call through ``recap_b200.Operator.attend`` (the
reference-facing API); one REFRESH precedes the steps.  With N GPUs the 24 heads are
split N ways (one process per GPU, no collective inside a SPARSE step): the layer call's
time is the max over ranks, so the scaling is strong.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's CPU path (the
oracle restatement, see oracle/cpu_baseline.py) instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

# BASELINE configs 4 (the headline), 2 and 3.  batch: the layer call's batch (CogVideoX runs
# its two guidance branches as batch 2, recap/models/cogvideox.py:17).
WORKLOADS = {
    "hunyuan720p_layer": dict(name="hunyuan720p_layer", label="HunyuanVideo-720p layer", grid=(33, 45, 80),
                              heads=24, dim=128, text=256, text_first=False, density=0.1, batch=1),
    "wan480p_layer": dict(name="wan480p_layer", label="Wan2.1-1.3B 480p layer", grid=(21, 30, 52), heads=12,
                          dim=128, text=0, text_first=False, density=0.2, batch=1),
    "cogvideox768_layer": dict(name="cogvideox768_layer", label="CogVideoX-1.5 768p layer, guidance batch 2",
                               grid=(11, 48, 85), heads=48, dim=64, text=226, text_first=True, density=0.15,
                               batch=2),
    # the 60 attention layers (20 double-stream + 40 single-stream blocks
    # attend jointly over [video | text] alike) of a 3072-wide HunyuanVideo DiT, random-init
    # Q/K/V and output projections, Ulysses sequence sharding around head-parallel attention
    "hunyuan720p_stack60": dict(name="hunyuan720p_stack60", label="HunyuanVideo-720p 60-layer attention stack",
                                grid=(33, 45, 80), heads=24, dim=128, text=256, text_first=False, density=0.1,
                                batch=1, layers=60, hidden=3072, schedule_steps=50, refresh_every=5),
}
WORKLOAD = WORKLOADS["hunyuan720p_layer"]
UNIT = "us/layer"


def metric_of(w: dict) -> str:
    return f"corrected sparse-attn us/layer call ({w['label']}, SPARSE step)"


METRIC = metric_of(WORKLOAD)


def head_slice(heads: int, world: int, rank: int) -> range:
    """This rank's heads: contiguous, the first heads % world ranks one more (12 heads over
    8 GPUs: 2/2/2/2/1/1/1/1)."""
    base, extra = divmod(heads, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default=WORKLOAD["name"],
                   help="BASELINE config 4 (default), 2 or 3")
    p.add_argument("--exchange", choices=["push", "p2p", "nccl"], default="push",
                   help="stack workload, the Ulysses exchange: a kernel of peer stores writing the projections "
                        "into the owners' receive buffers and the attention epilogue storing rows into the "
                        "owners' shards (push); the layout pass reading the ranks' projections in place over "
                        "NVLink (p2p); or NCCL all_to_all_single around the call (nccl)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-copy-streams", type=int, default=3,
                   help="host-to-device copy streams of the e2e leg (the three inputs share them)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true", help="skip the CPU oracle check of the last timed output")
    p.add_argument("--profile-steps", type=int, default=0,
                   help="extra steps after the timed region; their per-kernel times are reported as "
                        "kernels_ms_extra_steps (the per-kernel times of the timed steps are always reported)")
    p.add_argument("--heads", type=int, default=None,
                   help="run only this many of the layer's heads (small cases for ncu captures)")
    p.add_argument("--kernel", choices=["select"], default=None,
                   help="time one kernel alone at the workload's shape instead of the layer call (select: "
                        "recap_pool_select on seeded pooled means, about 45 MB on the device)")
    return p.parse_args()


# ----------------------------------------------------------------------------- data


def synth_qkv(grid, heads: range, dim: int, text: int, text_first: bool, seed: int, device, rank: int = 16,
              noise: float = 0.5, batch: int = 1):
    """Seeded Q/K/V [batch, len(heads), S, dim] bf16 with per-frame spatially smooth low-rank
    structure (sum of 4 low-frequency cosines per factor, per-frame phase drift) plus
    noise; text tokens N(0,1).  Generated per (batch, head) on the device."""
    T, H, W = grid
    nv = T * H * W
    tt = torch.arange(T, dtype=torch.float32, device=device).view(T, 1, 1)
    yy = (torch.arange(H, dtype=torch.float32, device=device) / H).view(1, H, 1)
    xx = (torch.arange(W, dtype=torch.float32, device=device) / W).view(1, 1, W)
    out = []
    for tensor in range(3):
        x = torch.empty(batch, len(heads), nv + text, dim, dtype=torch.bfloat16, device=device)
        for bi, i, h in ((bi, i, h) for bi in range(batch) for i, h in enumerate(heads)):
            g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + tensor * 10_007 + h + 100_003 * bi)
            u = torch.randn(rank, dim, generator=g, device=device) / math.sqrt(rank)
            amp = torch.randn(rank, 4, generator=g, device=device)
            ky = torch.randint(-2, 3, (rank, 4), generator=g, device=device).float()
            kx = torch.randint(-2, 3, (rank, 4), generator=g, device=device).float()
            ph = torch.rand(rank, 4, generator=g, device=device) * 2 * math.pi
            dr = (torch.rand(rank, 4, generator=g, device=device) - 0.5) * 0.6
            f = torch.zeros(rank, T, H, W, device=device)
            for c in range(4):
                v = lambda a: a[:, c].view(rank, 1, 1, 1)  # noqa: E731
                f += v(amp) * torch.cos(2 * math.pi * (v(ky) * yy + v(kx) * xx) + v(ph) + v(dr) * tt)
            vid = f.reshape(rank, nv).T @ u + noise * torch.randn(nv, dim, generator=g, device=device)
            txt = torch.randn(text, dim, generator=g, device=device)
            x[bi, i] = torch.cat([txt, vid]) if text_first else torch.cat([vid, txt])
        out.append(x)
    return out


def perturbed(xs, seed: int, device, eps: float = 0.05):
    g = torch.Generator(device=device).manual_seed(seed)
    return [(x.float() + eps * torch.randn(x.shape, generator=g, device=device)).to(x.dtype) for x in xs]


# ----------------------------------------------------------------------------- helpers


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    # NVML clock-event reason bits (nvmlClocksEventReason*)
    NVML_REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
                    0x4: "sw_power_cap"}

    def __init__(self, bus_id: str | None = None):
        # nvidia-smi's --id reads a bare index as a physical GPU index, which is not this
        # process's GPU under CUDA_VISIBLE_DEVICES: name the device by its PCI bus id
        if bus_id is None:
            prop = torch.cuda.get_device_properties(torch.cuda.current_device())
            bus_id = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
        self.bus_id = bus_id
        self.proc = None
        self.skip = 0
        self.nvml = None      # NVML handle of this process's GPU, for polling while it drains
        self.polled = []      # (sm_mhz, max_mhz, reason bits) taken by poll_until()
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"recap_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.bus_id}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            # nvidia-smi takes a while to start: begin the timed region once it samples,
            # and count only the samples taken from then on
            t0 = time.time()
            while time.time() - t0 < 5.0:
                lines = self.path.read_text().count("\n")
                if lines >= 1:
                    self.skip = lines
                    break
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def _nvml_handle(self):
        if self.nvml is None:
            try:
                import pynvml
                pynvml.nvmlInit()
                self.nvml = pynvml.nvmlDeviceGetHandleByPciBusId(self.bus_id.encode())
            except Exception:
                self.nvml = False
        return self.nvml or None

    def poll_until(self, event: "torch.cuda.Event") -> None:
        """Sample SM clock and clock-event reasons through NVML every few ms until `event`
        completes: a timed region shorter than nvidia-smi's sampling period (a few short
        steps on many GPUs) still gets samples taken while its kernels run."""
        h = self._nvml_handle()
        while not event.query():
            if h is not None:
                try:
                    import pynvml
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                    bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.polled.append((float(sm), float(mx), int(bits)))
                except Exception:
                    h = None
            time.sleep(0.002)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        try:
            rows = [r.split(",") for r in self.path.read_text().strip().splitlines()[self.skip:]]
        except Exception:
            rows = []
            if not self.polled:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = sorted(float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit())
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            if len(r) < 9:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        for smv, mxv, bits in self.polled:
            sm.append(smv)
            mx.append(mxv)
            for bit, name in self.NVML_REASONS.items():
                if bits & bit:
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def kept_tile_flops(partition: torch.Tensor, S: int, nv: int, dim: int) -> float:
    """sum over banks and kept 128x128 tiles of 4 * m_i * n_j * d with the real token counts
    of the blocks on the reordered sequence."""
    banks = partition.shape[0] * partition.shape[1]
    nb = partition.shape[-1]
    NB = (S + 127) // 128
    shared = nv % 128 != 0 and S > nv
    ds = nb - 1 if shared else nb
    counts = torch.full((NB,), 128.0, dtype=torch.float64)
    counts[-1] = S - 128 * (NB - 1)
    part = partition.reshape(banks, nb, nb).to(torch.float64).cpu()
    mask = torch.zeros(banks, NB, NB, dtype=torch.float64)
    mask[:, :nb, :nb] = part
    mask[:, ds:, :] = 1
    mask[:, :, ds:] = 1
    per_bank = torch.einsum("bij,i,j->b", mask, counts, counts)
    return float(per_bank.sum()) * 4 * dim


def peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d["bf16_tflops_sustained"],
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def traffic_per_launch() -> float | None:
    """DRAM bytes of one sparse-step launch at the bench workload, from the committed ncu
    summary (profiles/sparse_step_hunyuan720p.json), or None."""
    path = REPO / "profiles" / "sparse_step_hunyuan720p.json"
    if not path.exists():
        return None
    try:
        return float(json.loads(path.read_text())["dram_bytes_per_launch_full_workload"])
    except Exception:
        return None


def end_to_end(op, host, steps: int, group, n_heads: int, total_heads: int, copy_streams: int = 3) -> dict:
    """The layer call through ``Operator.attend`` with host-resident inputs and outputs:
    every step copies its Q/K/V from pinned host memory to the device and its output back.
    Double-buffered like a serving loop: the host-to-device copy of step i+1 and the
    device-to-host copy of step i run on their own streams while step i computes (the
    copy engines and the SMs work at once).  The serial figure (copy in, compute, copy
    out, one after another on one stream) is reported beside it."""
    import torch.distributed as dist

    dev = torch.device("cuda", torch.cuda.current_device())
    comp = torch.cuda.current_stream()
    # one copy stream per input tensor: the three host-to-device copies run on separate
    # copy engines at once
    h2d_s = [torch.cuda.Stream() for _ in range(max(1, min(copy_streams, len(host[0]))))]
    d2h_s = torch.cuda.Stream()
    dev_in = [[torch.empty_like(t, device=dev) for t in host[0]] for _ in range(2)]
    out_host = [torch.empty(host[0][0].shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]

    def timed(fn) -> float:
        torch.cuda.synchronize()
        if group is not None:
            dist.barrier(group=group)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        fn(e0)
        e1.record(comp)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if group is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item()) / steps * 1000.0

    def serial(start):
        for i in range(steps):
            for dst, src in zip(dev_in[0], host[i % 2]):
                dst.copy_(src, non_blocking=True)
            out_host[0].copy_(op.attend(0, *dev_in[0]), non_blocking=True)

    def pipelined(start):
        n_in = len(host[0])
        loaded = [[torch.cuda.Event() for _ in range(n_in)] for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]
        computed = [torch.cuda.Event() for _ in range(2)]

        def copy_in(i):
            b = i % 2
            for j, (dst, src) in enumerate(zip(dev_in[b], host[i % 2])):
                st = h2d_s[j % len(h2d_s)]
                with torch.cuda.stream(st):
                    st.wait_event(start)
                    st.wait_event(consumed[b])  # step i-2 has finished reading this buffer
                    dst.copy_(src, non_blocking=True)
                    loaded[b][j].record(st)

        copy_in(0)
        for i in range(steps):
            b = i % 2
            if i + 1 < steps:
                copy_in(i + 1)
            for ev in loaded[b]:
                comp.wait_event(ev)
            out = op.attend(0, *dev_in[b])
            consumed[b].record(comp)
            computed[b].record(comp)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(computed[b])
                out_host[b].copy_(out, non_blocking=True)
            out.record_stream(d2h_s)
        comp.wait_stream(d2h_s)
        for st in h2d_s:
            comp.wait_stream(st)

    serial(None)  # warm the copy paths
    pipelined(torch.cuda.Event())
    torch.cuda.synchronize()
    t_serial = timed(serial)
    t_pipe = timed(pipelined)
    # bytes of all ranks: this rank's per head, times the layer's heads
    h2d = sum(t.numel() * t.element_size() for t in host[0]) // n_heads * total_heads
    d2h = out_host[0].numel() * 2 // n_heads * total_heads
    return {"value": round(t_pipe, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "pipeline": f"double-buffered: H2D of step i+1 ({len(h2d_s)} copy stream(s) for the three inputs) and "
                        "D2H of step i on copy streams during step i",
            "serial_value": round(t_serial, 1)}


def workload_config(w: dict, world: int) -> dict:
    """The ``config`` of both arms' JSON lines."""
    nv = w["grid"][0] * w["grid"][1] * w["grid"][2]
    nb = (nv + 127) // 128
    S = nv + w["text"]
    in_gb = 3 * w["batch"] * w["heads"] * S * w["dim"] * 2 / 1e9
    split = [len(head_slice(w["heads"], world, r)) for r in range(world)]
    par = f"heads/{world}" if len(set(split)) == 1 else f"heads/{world} uneven " + "/".join(map(str, split))
    return {"workload": w["name"], "batch": w["batch"], "heads": w["heads"], "head_dim": w["dim"],
            "video_tokens": nv, "text_tokens": w["text"], "seq_len": S, "key_blocks": nb,
            "keep": max(1, round(w["density"] * nb)), "parallelism": par, "bank": "HBM",
            "l2": f"inputs {in_gb:.2f} GB per step > 126 MB L2 (no flush needed)"}


def selection_roofline(w: dict, n_heads: int, refresh_times: dict, hbm_gbs: float) -> dict:
    """HBM figures of the selection at a REFRESH (this rank's banks).  B_sel counts the
    algorithmic bytes of pooling and top-k: the Q and K video rows read once (bf16), the
    pooled means written (fp32) and the kept indices (4 bytes each).  The pooling runs
    inside the layout pass, which also writes the reordered operands of the attention
    kernels, so B_sel over gather + select time is a lower bound of the selection's rate;
    the layout pass's own bytes and rate are reported beside it."""
    nv = w["grid"][0] * w["grid"][1] * w["grid"][2]
    S = nv + w["text"]
    d = w["dim"]
    banks = n_heads * w["batch"]
    nb = (nv + 127) // 128
    keep = max(1, round(w["density"] * nb))
    s_pad = 128 * ((S + 127) // 128)
    b_sel = 2 * banks * nv * d * 2 + 2 * banks * nb * d * 4 + banks * nb * keep * 4
    t_g = sum(refresh_times.get("recap_layout_gather", [0.0]))
    t_s = sum(refresh_times.get("recap_pool_select", [0.0]))
    # layout pass: read Q, K, V native; write Q, K, V^T and the centred K^T (bf16), the
    # three pooled means and the bf16 mean copies
    b_gather = 3 * banks * S * d * 2 + 4 * banks * s_pad * d * 2 + 3 * banks * nb * d * 4
    out = {"algorithmic_bytes": b_sel, "kernels_ms": {"recap_layout_gather": round(t_g, 4),
                                                      "recap_pool_select": round(t_s, 4)},
           "peak_gbs": hbm_gbs, "gather_pass_bytes": b_gather}
    if t_g + t_s > 0:
        out["achieved_gbs"] = round(b_sel / ((t_g + t_s) * 1e-3) / 1e9, 1)
        out["frac"] = round(out["achieved_gbs"] / hbm_gbs, 4)
    if t_g > 0:
        out["gather_pass_gbs"] = round(b_gather / (t_g * 1e-3) / 1e9, 1)
        out["gather_pass_frac"] = round(out["gather_pass_gbs"] / hbm_gbs, 4)
    return out


def parity_leg(w: dict, layout, hx: dict, basis, part0, part2, keep: bool, out_rows: dict, oracle_qblocks) -> dict:
    """The last timed SPARSE output of the sampled banks against the block oracle on the
    CPU (oracle/block_oracle.py), replaying the REFRESH on x0, the revalidating REFRESH on
    x2 and the SPARSE step on the last timed inputs."""
    from oracle import block_oracle as bo

    t0 = time.perf_counter()
    perm = layout.permutation
    orc_ = bo.BlockOracle(perm, w["text"], w["text_first"], w["density"], qblocks=oracle_qblocks)
    fwd = orc_.fwd
    nv = layout.video_tokens
    mism = bo.selection_mismatches(part0, hx["x0"][0][:, fwd], hx["x0"][1][:, fwd], w["density"], nv)
    orc_.refresh(*hx["x0"], basis=basis, partition=part0)
    orc_.step = 1
    if not keep:
        mism += bo.selection_mismatches(part2, hx["x2"][0][:, fwd], hx["x2"][1][:, fwd], w["density"], nv)
    orc_.refresh(*hx["x2"], decision=keep, new_partition=None if keep else part2)
    orc_.step = 2
    exp = orc_.sparse(*hx["last"])
    got = torch.cat([out_rows[qb].reshape(-1) for qb in sorted(exp)])
    ref = torch.cat([exp[qb].reshape(-1) for qb in sorted(exp)])
    c = bo.compare_bf16(got, ref)
    return {"max_abs": round(c["max_abs"], 5), "mean_rel": round(c["mean_rel"], 6),
            "elements": c["n"], "elements_over_2e-2": c["n_over_2e-2"],
            "max_bf16_ulps_over_2e-2": round(c["max_ulps_over_2e-2"], 3), "max_abs_ref": round(c["max_abs_ref"], 3),
            "selection_mismatches_beyond_ties": mism, "banks": hx["banks"], "query_blocks": len(exp),
            "cpu_s": round(time.perf_counter() - t0, 1),
            "checked": "last timed SPARSE output, sampled banks x query blocks (every dense block), "
                       "against the CPU block oracle replaying REFRESH(x0) -> REFRESH(x2) -> SPARSE"}


# ----------------------------------------------------------------------------- our arm


def run_ours(args) -> None:
    import torch.distributed as dist

    from recap_b200 import REFRESH, SPARSE, Operator, OperatorConfig
    from recap_b200.sparse import Layout, SparseGeometry, hilbert_permutation

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        group = dist.group.WORLD
    w = dict(WORKLOADS[args.workload])
    if w.get("layers"):
        return run_stack(args, w, world, rank, dev, group)
    if args.heads:
        w["heads"] = int(args.heads)
        w["name"] = f'{w["name"]}_{args.heads}heads'
    H = w["heads"]
    if H < world:
        raise SystemExit(f"{H} heads cannot give each of {world} GPUs one")
    hs = head_slice(H, world, rank)
    perm = hilbert_permutation(w["grid"])
    layout = Layout.from_permutation(perm, text_tokens=w["text"], text_first=w["text_first"])
    geo = SparseGeometry.build(layout, 128)
    cfg = OperatorConfig(head_density=w["density"])
    op = Operator.build(cfg, geo, n_layers=1, process_group=group)
    nv = layout.video_tokens
    S = nv + w["text"]
    d = w["dim"]

    x0 = synth_qkv(w["grid"], hs, d, w["text"], w["text_first"], seed=0, device=dev, batch=w["batch"])
    op.begin_step(0, REFRESH)
    op.attend(0, *x0)
    torch.cuda.synchronize()
    x1 = perturbed(x0, 1, dev)
    x2 = perturbed(x1, 2, dev)
    check = rank == 0 and not args.no_parity
    hx: dict = {}
    if check:
        # two banks of rank 0 (its first and last head) for the parity leg, on the host
        sb = sorted({0, len(hs) - 1})
        hx = {"banks": sb, **{n: [t[0, sb].float().cpu() for t in x] for n, x in (("x0", x0), ("x1", x1), ("x2", x2))}}
        hx["part0"] = op.banks[0][0].partition[0, sb].cpu().clone()
        hx["basis"] = op.layers[0][0].basis[sb].cpu().clone()
    part0_dev = op.banks[0][0].partition.clone()
    del x0
    inputs = [x1, x2]

    # refresh timing: a revalidating refresh on x2, device time from a common start (the
    # ranks meet at a barrier first), max over ranks; per-call times beside it.  The first
    # revalidating call of the process also makes the caching allocator's first allocations
    # at its shapes (host stalls of 10-80 ms measured before its first launch), so that call
    # runs untimed first; a second revalidating refresh on the same inputs leaves the same
    # state (the same partition is kept, the same refinement and coarse LSE are written).
    op.begin_step(1, REFRESH)
    op.attend(0, *x2)
    torch.cuda.synchronize()
    op.drain_validation()
    op.begin_step(1, REFRESH)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if group is not None:
        # the revalidating refresh all-reduces its overlap counts: have NCCL set up the
        # int64 all-reduce before the timed region
        dist.all_reduce(torch.zeros(2, dtype=torch.int64, device=dev), group=group)
    torch.cuda.synchronize()
    if group is not None:
        dist.barrier(group=group)
    op.launches.timing = True
    t0.record()
    op.attend(0, *x2)
    t1.record()
    torch.cuda.synchronize()
    op.launches.timing = False
    refresh_times = op.launches.take_times()
    refresh_t = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(refresh_t, op=dist.ReduceOp.MAX, group=group)
    refresh_ms = float(refresh_t.item())
    op.drain_validation()
    keep = bool(torch.equal(op.banks[0][0].partition, part0_dev))
    if check:
        hx["part2"] = op.banks[0][0].partition[0, hx["banks"]].cpu().clone()
    del part0_dev

    op.begin_step(2, SPARSE)
    for i in range(args.warmup):
        op.attend(0, *inputs[i % 2])
    torch.cuda.synchronize()
    if group is not None:
        dist.barrier(group=group)
    launches_before = op.launches.count
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    # per-launch events inside the timed steps (a few microseconds each): the kernel breakdown
    # and the roofline describe the same steps, clocks and power state as the headline figure
    op.launches.timing = True
    op.launches.take_times()
    with ClockSampler() as clk:
        torch.cuda.synchronize()
        start.record()
        for i in range(args.steps):
            out = op.attend(0, *inputs[i % 2])
        end.record()
        clk.poll_until(end)  # the host queued every step: sample while the GPU runs them
        torch.cuda.synchronize()
    op.launches.timing = False
    times = op.launches.take_times()
    if group is not None:
        dist.barrier(group=group)
    gpu_launches = op.launches.count - launches_before
    elapsed = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX, group=group)
    ms_per_step = float(elapsed.item()) / args.steps
    out_rows = None
    if check:
        from oracle.block_oracle import BlockOracle, sample_qblocks

        oracle_qblocks = sample_qblocks(nv, S, 8)
        fwd = BlockOracle(layout.permutation, w["text"], w["text_first"], w["density"], qblocks=[]).fwd
        sel = out[0, hx["banks"]]
        out_rows = {qb: sel[:, fwd[qb * 128: min(S, (qb + 1) * 128)].to(dev)].float().cpu() for qb in oracle_qblocks}
        hx["last"] = hx["x1"] if (args.steps - 1) % 2 == 0 else hx["x2"]
    del out

    kernels_ms = {k: sum(v) / len(v) for k, v in times.items()}
    kernels_extra = None
    if args.profile_steps > 0:
        op.launches.timing = True
        for i in range(args.profile_steps):
            op.attend(0, *inputs[i % 2])
        kernels_extra = {k: round(sum(v) / len(v), 4) for k, v in op.launches.take_times().items()}
        op.launches.timing = False
    fmha_ms = kernels_ms.get("recap_sparse_step")
    flops = kept_tile_flops(op.banks[0][0].partition, S, nv, d)
    flops_t = torch.tensor([flops], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(flops_t, group=group)
    pk = peaks()
    achieved = flops / (fmha_ms * 1e-3) / 1e12 if fmha_ms else None
    traffic = traffic_per_launch()
    if traffic is not None:
        # the committed figure is for all 24 heads of the default workload on one GPU
        traffic = traffic * len(hs) / WORKLOAD["heads"] if w["name"] == WORKLOAD["name"] else None

    # end to end through the API with host buffers
    e2e = None
    if not args.no_e2e:
        host = [[t.cpu().pin_memory() for t in xs] for xs in inputs]
        e2e = end_to_end(op, host, args.steps, group, len(hs), H, copy_streams=args.e2e_copy_streams)
        del host
    op.check_device_status()

    parity = None
    if check:
        parity = parity_leg(w, layout, hx, hx["basis"], hx["part0"], hx["part2"], keep, out_rows, oracle_qblocks)
    del hx, out_rows

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.cpu_baseline import time_sparse_sample

        cpu = time_sparse_sample(op, inputs[0], layout, w)

    if rank == 0:
        dense_flops = 4.0 * S * S * d * H * w["batch"]
        line = {
            "metric": metric_of(w), "value": round(ms_per_step * 1000.0, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded smooth low-rank (rank 16) + 0.5 noise Q/K/V, 0.05 perturbation per step",
            "config": workload_config(w, world),
            "dense_equiv_tflops": round(dense_flops / (ms_per_step * 1e-3) / 1e12, 1),
            "refresh_us": round(refresh_ms * 1000.0, 1),
            "refresh_timed": "a revalidating REFRESH call after an untimed one on the same inputs",
            "refresh_kernels_ms": {k: round(sum(v), 4) for k, v in refresh_times.items()},
            "refresh_rerank": not keep,
            "selection": selection_roofline(w, len(hs), refresh_times, pk["hbm_gbs"]),
            "kernels_ms": {k: round(v, 4) for k, v in kernels_ms.items()},
            "kernels_ms_of": "the timed steps (per-launch events on the launching stream)",
            **({"kernels_ms_extra_steps": kernels_extra} if kernels_extra else {}),
            "roofline": {
                "kernel": "recap_sparse_step (block-sparse FMHA + corrected merge)",
                "bound": "tensor", "achieved": round(achieved, 1) if achieved else None,
                "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops_sustained"], 4) if achieved else None,
                "peak_kind": f"bf16 sustained ({pk['source']})",
                "algorithmic_flops_per_launch": flops,
                "traffic": traffic,
            },
            "gpu_launches": gpu_launches,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "parity": parity,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if group is not None:
        dist.barrier(group=group)
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- the 60-layer stack


def stack_hidden(w: dict, tokens: range, hidden: int, seed: int, device, rank: int = 16, noise: float = 0.5):
    """Seeded hidden states ``[len(tokens), hidden]`` bf16 of the given sequence positions:
    the video tokens a per-frame spatially smooth rank-16 field (as ``synth_qkv``) times
    random directions plus noise, the text tokens N(0, 1).  Every rank draws the same field
    and directions and keeps its own tokens."""
    T, H, W = w["grid"]
    nv = T * H * W
    g = torch.Generator(device=device).manual_seed(seed)
    u = torch.randn(rank, hidden, generator=g, device=device) / math.sqrt(rank)
    tt = torch.arange(T, dtype=torch.float32, device=device).view(T, 1, 1)
    yy = (torch.arange(H, dtype=torch.float32, device=device) / H).view(1, H, 1)
    xx = (torch.arange(W, dtype=torch.float32, device=device) / W).view(1, 1, W)
    f = torch.zeros(rank, T, H, W, device=device)
    amp = torch.randn(rank, 4, generator=g, device=device)
    ky = torch.randint(-2, 3, (rank, 4), generator=g, device=device).float()
    kx = torch.randint(-2, 3, (rank, 4), generator=g, device=device).float()
    ph = torch.rand(rank, 4, generator=g, device=device) * 2 * math.pi
    dr = (torch.rand(rank, 4, generator=g, device=device) - 0.5) * 0.6
    for c in range(4):
        v = lambda a: a[:, c].view(rank, 1, 1, 1)  # noqa: E731
        f += v(amp) * torch.cos(2 * math.pi * (v(ky) * yy + v(kx) * xx) + v(ph) + v(dr) * tt)
    f = f.reshape(rank, nv)
    idx = torch.arange(tokens.start, tokens.stop, device=device)
    vid = idx[idx < nv] if not w["text_first"] else idx[idx >= w["text"]] - w["text"]
    out = torch.empty(len(tokens), hidden, dtype=torch.bfloat16, device=device)
    gn = torch.Generator(device=device).manual_seed(seed * 7919 + tokens.start)
    is_vid = (idx < nv) if not w["text_first"] else (idx >= w["text"])
    out[is_vid] = (f[:, vid].T @ u + noise * torch.randn(len(vid), hidden, generator=gn, device=device)).to(out.dtype)
    n_txt = int((~is_vid).sum())
    if n_txt:
        out[~is_vid] = torch.randn(n_txt, hidden, generator=gn, device=device).to(out.dtype)
    return out


class AttentionStack:
    """``layers`` joint-attention layers of width ``hidden``: per layer
    x += heads_to_seq(attend(seq_to_heads(x W_qkv))) W_o, with ``x`` sharded by sequence
    over the ranks and the attention sharded by head (Ulysses).  Random-init projections
    (the benchmark has no checkpoint); the attention is ``recap_b200.Operator.attend``.
    ``timing`` records CUDA events around each phase of every layer."""

    PHASES = ("qkv_projection", "all_to_all_seq_to_heads", "attention", "all_to_all_heads_to_seq",
              "out_projection")

    def __init__(self, op, w: dict, world: int, group, device, exchange: str = "nccl"):
        from recap_b200.ulysses import PeerBuffer, ShardedIO, check_split

        self.op, self.world, self.group = op, world, group
        self.exchange = exchange if world > 1 else "nccl"
        self.heads, self.dim, self.hidden = w["heads"], w["dim"], w["hidden"]
        self.S = w["grid"][0] * w["grid"][1] * w["grid"][2] + w["text"]
        self.s, self.h = check_split(self.S, self.heads, world)
        if self.heads * self.dim != self.hidden:
            raise ValueError("heads x head_dim must equal the hidden width")
        hd = self.heads * self.dim
        g = torch.Generator(device=device).manual_seed(1234)
        bf = torch.bfloat16
        self.w_qkv = [(torch.randn(self.hidden, 3 * hd, generator=g, device=device) / math.sqrt(self.hidden)).to(bf)
                      for _ in range(w["layers"])]
        self.w_o = [(torch.randn(hd, self.hidden, generator=g, device=device) * (0.5 / math.sqrt(hd))).to(bf)
                    for _ in range(w["layers"])]
        self.timing = False
        self.events: list[list] = []
        self.io = None
        self.peers: list = []
        if self.exchange in ("p2p", "push"):
            # the attention output of every rank, reachable by all; p2p: the projections too;
            # push: each rank's receive buffer of its heads' projections
            self.peer_out = PeerBuffer(self.s * hd * 2, group, device)
            self.peers.append(self.peer_out)
            if self.exchange == "p2p":
                self.peer_qkv = PeerBuffer(self.s * 3 * hd * 2, group, device)
                self.peers.append(self.peer_qkv)
                self.io = ShardedIO(self.peer_qkv, self.peer_out, self.heads, self.dim, self.S)
            else:
                self.peer_recv = PeerBuffer(self.S * 3 * self.h * self.dim * 2, group, device)
                self.peers.append(self.peer_recv)
                self.qkv_local = torch.empty(self.s, 3, self.heads, self.dim, dtype=bf, device=device)
                self.io = ShardedIO(None, self.peer_out, self.heads, self.dim, self.S, recv=self.peer_recv)
            self.flag = torch.zeros(1, device=device)

    def close(self) -> None:
        for p in self.peers:
            p.close()
        self.peers = []
        self.io = None

    def _meet(self) -> None:
        """Every rank's writes so far are done before any rank goes on (a one-element
        all-reduce on the stream: its kernel starts after this rank's earlier work and ends
        after every rank's)."""
        import torch.distributed as dist

        dist.all_reduce(self.flag, group=self.group)

    def _mark(self, marks: list) -> None:
        if self.timing:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            marks.append(e)

    def step(self, x: torch.Tensor) -> torch.Tensor:
        """One denoising step's attention layers on this rank's tokens ``[s, hidden]``."""
        from recap_b200.ulysses import heads_to_seq, seq_to_heads

        if self.io is not None:
            return self._step_p2p(x)
        for layer in range(len(self.w_qkv)):
            marks: list = []
            self._mark(marks)
            qkv = (x @ self.w_qkv[layer]).view(self.s, 3, self.heads, self.dim)
            self._mark(marks)
            q, k, v = seq_to_heads(qkv, self.world, self.group)
            self._mark(marks)
            o = self.op.attend(layer, q, k, v)
            self._mark(marks)
            y = heads_to_seq(o, self.world, self.group)
            self._mark(marks)
            x = x + y @ self.w_o[layer]
            self._mark(marks)
            if self.timing:
                self.events.append(marks)
        return x

    def _step_p2p(self, x: torch.Tensor) -> torch.Tensor:
        """The layer with the exchange in place: the projection writes this rank's shard of
        the shared buffer, the layout pass reads every rank's shard of this rank's heads
        over NVLink, and the attention epilogue stores each output row into the shard of
        the rank that owns the token."""
        io = self.io
        push = self.exchange == "push"
        qkv4 = self.qkv_local if push else io.local_qkv()
        qkv = qkv4.view(self.s, 3 * self.heads * self.dim)
        y = io.local_out()
        for layer in range(len(self.w_qkv)):
            marks: list = []
            self._mark(marks)
            torch.matmul(x, self.w_qkv[layer], out=qkv)
            self._mark(marks)
            if push:
                # the owners finished reading their receive buffers before the last meeting
                io.push(qkv4)
            self._meet()  # every shard written (pushed) before any rank reads
            self._mark(marks)
            self.op.attend_sharded(layer, io)
            self._mark(marks)
            self._meet()  # every output row stored, every shard read
            self._mark(marks)
            x = x + y @ self.w_o[layer]
            self._mark(marks)
            if self.timing:
                self.events.append(marks)
        return x

    def take_phases(self) -> dict:
        """Milliseconds per phase summed over the recorded layers (synchronises)."""
        torch.cuda.synchronize()
        tot = {p: 0.0 for p in self.PHASES}
        for marks in self.events:
            for i, p in enumerate(self.PHASES):
                tot[p] += marks[i].elapsed_time(marks[i + 1])
        self.events = []
        return tot


def run_stack(args, w: dict, world: int, rank: int, dev, group) -> None:
    """BASELINE config 5 on N GPUs: steps of the 60-layer stack.  One REFRESH step warms
    up, one revalidating REFRESH step and ``--steps`` SPARSE steps are timed (device time,
    max over ranks); the 50-step schedule with a refresh every 5th step is reported as
    10 x REFRESH + 40 x SPARSE from those measurements."""
    import torch.distributed as dist

    from recap_b200 import REFRESH, SPARSE, Operator, OperatorConfig
    from recap_b200.sparse import Layout, SparseGeometry, hilbert_permutation

    layout = Layout.from_permutation(hilbert_permutation(w["grid"]), text_tokens=w["text"],
                                     text_first=w["text_first"])
    op = Operator.build(OperatorConfig(head_density=w["density"]), SparseGeometry.build(layout, 128),
                        n_layers=w["layers"], process_group=group)
    stack = AttentionStack(op, w, world, group, dev, exchange=args.exchange)
    mine = range(rank * stack.s, (rank + 1) * stack.s)
    xs = [stack_hidden(w, mine, w["hidden"], seed=s, device=dev) for s in (0, 1, 2)]

    def timed(kind: str, n: int, first_step: int, phases: bool = False):
        torch.cuda.synchronize()
        if group is not None:
            dist.barrier(group=group)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        stack.timing = phases
        e0.record()
        for i in range(n):
            op.begin_step(first_step + i, kind)
            stack.step(xs[(first_step + i) % 3])
        e1.record()
        torch.cuda.synchronize()
        stack.timing = False
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if group is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item()) / n

    with torch.no_grad():
        if group is not None:
            dist.all_reduce(torch.zeros(2, dtype=torch.int64, device=dev), group=group)
        timed(REFRESH, 1, 0)  # first refresh: selection, banks of every layer
        refresh_ms = timed(REFRESH, 1, 1)  # revalidating refresh of every layer
        op.drain_validation()
        step = 2
        if args.warmup:
            timed(SPARSE, args.warmup, step)
            step += args.warmup
        launches_before = op.launches.count
        with ClockSampler() as clk:
            torch.cuda.synchronize()
            sparse_ms = timed(SPARSE, args.steps, step)
        gpu_launches = op.launches.count - launches_before
        step += args.steps
        op.launches.timing = True
        timed(SPARSE, 1, step, phases=True)
        phases = stack.take_phases()
        ktimes = {k: sum(v) for k, v in op.launches.take_times().items()}
        op.launches.timing = False
        op.check_device_status()
        stack.close()
    total = sum(phases.values())
    a2a = phases["all_to_all_seq_to_heads"] + phases["all_to_all_heads_to_seq"]
    n_refresh = -(-w["schedule_steps"] // w["refresh_every"])
    schedule_s = (n_refresh * refresh_ms + (w["schedule_steps"] - n_refresh) * sparse_ms) / 1000.0
    if rank == 0:
        line = {
            "metric": f"corrected sparse-attn ms per denoising step ({w['label']}, SPARSE step)",
            "value": round(sparse_ms, 2), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(sparse_ms, 3), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded smooth low-rank (rank 16) + 0.5 noise hidden states, random-init projections",
            "config": {"workload": w["name"], "layers": w["layers"], "hidden": w["hidden"], "heads": w["heads"],
                       "head_dim": w["dim"], "seq_len": stack.S, "keep": max(1, round(w["density"] * -(-(stack.S - w["text"]) // 128))),
                       "parallelism": f"ulysses sequence/{world} + heads/{world}", "exchange": stack.exchange,
                       "bank": "HBM",
                       "l2": "per-layer inputs > 126 MB L2 (no flush needed)"},
            "us_per_layer": round(sparse_ms * 1000.0 / w["layers"], 1),
            "refresh_step_ms": round(refresh_ms, 2),
            "schedule_s": round(schedule_s, 2),
            "schedule": f"{w['schedule_steps']} steps, REFRESH every {w['refresh_every']}th: "
                        f"{n_refresh} x REFRESH + {w['schedule_steps'] - n_refresh} x SPARSE, from the measured steps",
            "phases_ms_per_step": {k: round(v, 3) for k, v in phases.items()},
            "all_to_all_share": round(a2a / total, 4) if total else None,
            "exchange_phases": {
                "nccl": "NCCL all_to_all_single with the layout copies around it",
                "push": "the peer-store kernel writing the projections plus the all-reduce that orders them; the "
                        "output rows go to their owners from the attention epilogue (in 'attention')",
                "p2p": "the two one-element all-reduces that order the ranks' buffer writes; the transfers "
                       "themselves run inside the layout pass and the attention epilogue"}[stack.exchange],
            "kernels_ms_per_step": {k: round(v, 3) for k, v in ktimes.items()},
            "gpu_launches": gpu_launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if group is not None:
        dist.barrier(group=group)
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- reference arm


def run_kernel_select(args) -> None:
    """``--kernel select``: the block selection (fp32 scores of every query-block x key-block
    pair of every bank and the exact top-k) alone, at the workload's banks, block count, head
    dimension and keep, on seeded pooled means (a shared low-rank part plus noise, so the
    scores of a row lie close together as they do for smooth video).  A small case for ncu:
    the means and the partition take about 45 MB at the default workload."""
    from recap_b200 import _lib as lib

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", 0)
    nv = w["grid"][0] * w["grid"][1] * w["grid"][2]
    d = w["dim"]
    banks = (args.heads or w["heads"]) * w["batch"]
    nb = (nv + 127) // 128
    keep = max(1, round(w["density"] * nb))
    g = torch.Generator().manual_seed(0)
    shared = torch.randn(nb, 16, generator=g) @ torch.randn(16, d, generator=g) / 4
    qm = (shared + 0.5 * torch.randn(banks, nb, d, generator=g)).to(dev)
    km = (shared + 0.5 * torch.randn(banks, nb, d, generator=g)).to(dev)
    part = torch.empty(banks, nb, nb, dtype=torch.bool, device=dev)
    st = lib.stream_handle(dev)

    def run():
        lib.call("recap_pool_select", lib.ptr(qm), lib.ptr(km), banks, nb, d, keep, 1 / math.sqrt(d), nv, 128,
                 lib.ptr(part), st)

    for _ in range(max(1, args.warmup)):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"kernel": "recap_pool_select", "ms": round(ms, 4), "steps": args.steps,
                      "config": {"workload": w["name"], "banks": banks, "key_blocks": nb, "head_dim": d,
                                 "keep": keep, "data": "seeded synthetic pooled means"},
                      "kept_per_row": round(float(part.sum(-1).float().mean()), 2)}), flush=True)


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle.cpu_baseline import reference_arm

    w = WORKLOADS[args.workload]
    if w.get("layers"):
        print(json.dumps({"impl": "reference", "unavailable": "the stack's CPU path is 60 calls of the "
                          "hunyuan720p_layer workload plus projections; its reference arm times one such layer"}),
              flush=True)
        return
    line = reference_arm(w, metric_of(w), UNIT, steps=args.steps, warmup=args.warmup,
                         config=workload_config(w, world))
    line.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup})
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    elif a.kernel == "select":
        run_kernel_select(a)
    else:
        run_ours(a)
