#!/usr/bin/env python
"""Benchmark of the B200 shift path: one position-shifted KV load turn per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--layout nhd]
    python bench.py --impl reference ...      # the reference's torch CPU path

A step is one shift turn of the BASELINE configuration (default c2, the
Qwen3-14B 30k edit turn: 28,608 tokens x 40 layers moved by delta +180, 8 KV
heads, head 128, bf16, block 16): every store row of the segment is read, K is
re-rotated, and K and V are scattered into the paged cache through a random
block table.  The inputs (5 GB of store + 5 GB of paged cache) are far larger
than the 126 MB L2, so no flush is needed between steps.

Under torchrun (N > 1) the turn is sharded by KV head as vLLM tensor
parallelism shards it: rank r holds heads [r*H/N, (r+1)*H/N) of the store and
the paged cache and moves only those; there is no data collective.  The only
NCCL traffic is one broadcast of the segment table at set-up.  `value` is the
whole turn's algorithmic bytes over the max-over-ranks device time.

Printed JSON keys beyond the driver's base contract:
  roofline      load kernel: algorithmic bytes per launch / its average launch
                duration over the timed region (region device time / the
                launches in it, back to back), against the measured HBM copy
                peak; isolated_turns: best and median of 10 single
                event-timed turns after the timed region
  e2e           the same turn through the public worker API (ShiftWorker.load)
                from host metadata: block table + descriptors copied from pinned
                host memory, tables + load kernels, the 4-byte status read back;
                loads are queued back to back and each status is read when the
                next load has been queued (the last one inside the timed region)
  cpu_baseline  the reference's torch CPU path on this host, bounded sample
  c3            (N=1, default config) the FP8 turn: kernel, e2e, roofline and a
                check against a torch restatement of dequantise/rotate/requantise
  c4            (N>1, default config) 64 sessions in one launch per rank at TP N
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "KV shift GB/s & ms/turn (30k-token Qwen3-14B shape) vs HBM peak at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
#: descriptor staging slots of the bench's own launchers: the host may queue
#: up to this many turns ahead of the GPU.  A host step was measured to stall
#: for 2.2 ms while an nvidia-smi poller (the clocks record) ran; with the
#: library's default of 4 slots that starved a 0.19 ms one-head turn, with 16
#: it was absorbed.  The GPU work per turn is the same either way; the e2e leg
#: uses the worker's launcher with the library default.
BENCH_SLOTS = 16


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--config", default="c2")
    ap.add_argument("--layout", default="nhd", choices=["nhd", "hnd", "split", "split_blocks"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--tile-tokens", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0, help="fewer layers (profiling cases)")
    ap.add_argument("--rank-share", type=int, default=0, metavar="N",
                    help="one GPU runs rank 0's head shard of an N-way split (profiling the "
                         "per-rank launch of an N-GPU run); the line reports that share")
    ap.add_argument("--no-save", action="store_true", help="skip the save-kernel timing")
    ap.add_argument("--no-alt", action="store_true", help="skip the TMA bulk-load timing")
    ap.add_argument("--no-host-tier", action="store_true",
                    help="skip the pinned-host store tier timing (N=1 only)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the c3 (N=1) / c4 (N>1) lines of the default run")
    ap.add_argument("--no-triton", action="store_true",
                    help="reference arm: skip the reference's Triton kernel on the GPU")
    return ap.parse_args()


def workload_config(cfg, world: int, layout: str, share: int = 0) -> dict:
    """The ``config`` object of both arms' lines: the workload only, identical in both.

    ``share`` > 1: one GPU runs rank 0's head shard of a ``share``-way split
    (a profiling case); the turn bytes are that shard's."""
    from marathon_b200.sharding import head_shard

    lo, hi = head_shard(cfg.heads, 0, share or world)
    if share:
        return {
            "workload": f"{cfg.name} {cfg.model} shift turn, rank 0's share of {share}",
            "layers": cfg.layers, "sessions": cfg.sessions,
            "tokens_shifted": cfg.shifted_tokens,
            "deltas": sorted({s.delta for segs in cfg.segments for s in segs}),
            "heads": cfg.heads, "heads_per_rank": hi - lo, "head_size": cfg.head_size,
            "block_size": cfg.block_size, "kv_dtype": cfg.dtype, "layout": layout,
            "parallelism": f"kv-head shard 1 of {share}, on one GPU",
            "turn_bytes": cfg.algorithmic_bytes(hi - lo),
            "l2": "inputs larger than L2 (store + paged cache per step >> 126 MB)",
        }
    return {
        "workload": f"{cfg.name} {cfg.model} shift turn", "layers": cfg.layers,
        "sessions": cfg.sessions, "tokens_shifted": cfg.shifted_tokens,
        "deltas": sorted({s.delta for segs in cfg.segments for s in segs}),
        "heads": cfg.heads, "heads_per_rank": hi - lo, "head_size": cfg.head_size,
        "block_size": cfg.block_size, "kv_dtype": cfg.dtype, "layout": layout,
        "parallelism": f"kv-head shard tp{world}", "turn_bytes": cfg.algorithmic_bytes(),
        "l2": "inputs larger than L2 (store + paged cache per step >> 126 MB)",
    }


# ----------------------------------------------------------------- helpers
def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def traffic_for(config: str, layout: str, units: int) -> float | None:
    """DRAM bytes per load launch from the committed ncu summary, scaled to ``units``."""
    p = ROOT / "profiles" / "traffic.json"
    try:
        rec = json.loads(p.read_text())[f"{config}/{layout}"]
        return rec["dram_bytes"] / rec["units"] * units
    except (OSError, KeyError, ValueError, ZeroDivisionError):
        return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons around a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.ident = None
        try:
            self.ident = f"GPU-{torch.cuda.get_device_properties(device).uuid}"
        except Exception:  # noqa: BLE001 - older torch: fall back to the ordinal
            self.ident = str(device.index or 0)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "-i", self.ident,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in csv.reader(io.StringIO(out)):
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                mx.append(float(row[2]))
            except ValueError:
                continue
            for name, val in zip(names, row[5:9], strict=True):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# --------------------------------------------------------- CPU baseline
def reference_shift_module():
    """The reference's own ``marathon.shift_kernels``, unmodified, from ``baseline/_ref``
    (installed by ``baseline/install_ref.py``); None when it is not installed."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "marathon" / "shift_kernels.py").is_file():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import marathon.shift_kernels as ref_sk

    return ref_sk


class CpuPath:
    """The reference's torch CPU path over ``cfg``'s first segment, one layer per call.

    bf16: the reference's own ``scatter_shifted_torch`` with tables from its own
    ``rope_shift(delta, head_size, inv_freq, "cpu")`` (``src/marathon/
    shift_kernels.py:68-84``, ``:141-159``), imported from ``baseline/_ref``
    (``kind`` "reference"); without that install, or for e4m3 (the reference
    has no scale handling), the restatement in ``oracle/torch_cpu_path.py``
    (``kind`` "port").  ``LAYERS`` distinct layers of store rows and paged
    cache are cycled, a working set far larger than the host's caches.
    """

    LAYERS = 4

    def __init__(self, cfg):
        from oracle import shift_oracle as O
        from oracle import torch_cpu_path as T

        self.T = T
        self.cfg = cfg
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        seg = cfg.segments[0][0]
        self.seg = seg
        self.n, h, d, bs = seg.length, cfg.heads, cfg.head_size, cfg.block_size
        blocks = -(-seg.dst_end // bs) + 16
        table = np.random.default_rng(0).permutation(blocks).astype(np.int64)
        self.slots = torch.from_numpy(O.slots(table, seg.dst_start, seg.dst_end, bs))
        self.inv = 1.0 / (cfg.theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        g = torch.Generator().manual_seed(0)
        self.fp8 = cfg.dtype == "e4m3"
        self.ref = None if self.fp8 else reference_shift_module()
        self.kind = "reference" if self.ref is not None else "port"
        if self.fp8:  # codes of the c3 distribution: values / per-layer scale, saturated
            self.k_scale = 0.05
            self.srcs = [(torch.randn(self.n, h, 2 * d, generator=g) * 20).clamp(-448, 448)
                         .to(torch.float8_e4m3fn) for _ in range(self.LAYERS)]
            self.kvs = [torch.zeros(blocks, bs, h, 2 * d, dtype=torch.float8_e4m3fn)
                        for _ in range(self.LAYERS)]
        else:
            self.srcs = [torch.randn(self.n, h, 2 * d, generator=g).to(torch.bfloat16)
                         for _ in range(self.LAYERS)]
            self.kvs = [torch.zeros(blocks, bs, h, 2 * d, dtype=torch.bfloat16)
                        for _ in range(self.LAYERS)]
        self.bs = bs
        self.i = 0
        self.run(layers=1, tokens=256)  # first touch

    @property
    def impl(self) -> str:
        if self.ref is not None:
            return "marathon.shift_kernels.scatter_shifted_torch (reference, baseline/_ref)"
        return "oracle/torch_cpu_path.py (restated torch path)"

    def run(self, layers: int = 1, tokens: int | None = None) -> tuple[float, int]:
        """``layers`` layer scatters of one turn (tables built once, as per load);
        returns (seconds, algorithmic bytes moved)."""
        n = self.n if tokens is None else min(tokens, self.n)
        d = self.cfg.head_size
        t0 = time.perf_counter()
        if self.ref is not None:
            shift = self.ref.rope_shift(self.seg.delta, d, self.inv, "cpu")
        else:
            from oracle import shift_oracle as O

            emb = self.T.emb_tables(torch.from_numpy(
                O.rope_tables([self.seg.delta], self.inv.numpy())[0]))
        for _ in range(layers):
            k = self.i % self.LAYERS
            self.i += 1
            src, kv, sl = self.srcs[k][:n], self.kvs[k], self.slots[:n]
            if self.ref is not None:
                self.ref.scatter_shifted_torch(src, kv, sl, self.bs, False, shift)
            elif self.fp8:
                self.T.scatter_layer_e4m3(src, kv, sl, self.bs, False, emb, self.k_scale)
            else:
                self.T.scatter_layer(src, kv, sl, self.bs, False, emb)
        return time.perf_counter() - t0, layers * n * self.cfg.bytes_per_token_layer()

    def sample(self, seconds: float) -> dict:
        done = moved = 0
        el = 0.0
        while el < seconds or done == 0:
            dt, b = self.run()
            el += dt
            moved += b
            done += 1
        return {"gbs": moved / el / 1e9, "seconds": el, "layers": done,
                "ms_per_layer": el / done * 1e3,
                "sample": f"{done} layer(s) of {self.cfg.name}: {self.n} tokens x "
                          f"{self.cfg.heads} heads x {2 * self.cfg.head_size} "
                          f"{self.cfg.dtype} each, {self.impl}, {self.threads} threads"}


def reference_triton(cfg, steps: int, warmup: int) -> dict:
    """The reference's unmodified Triton kernel on this GPU, one launch per layer.

    ``marathon.shift_kernels.scatter_shifted`` (``src/marathon/shift_kernels.py:
    162-210``) from ``baseline/_ref``: per turn, the tables of the load's delta
    (``rope_shift`` on the device) and one ``_shift_scatter_kernel`` launch per
    layer over the store rows, with the destination slots already on the
    device.  CUDA events around whole turns.
    """
    ref_sk = reference_shift_module()
    if ref_sk is None or not getattr(ref_sk, "HAVE_TRITON", False):
        return {"unavailable": "the reference package or Triton is not importable"}
    from marathon_b200.workloads import build

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = build(cfg, dev)
    r = wl.runs[0]
    bt = r.block_table.long()
    pos = torch.arange(r.paged_start, r.paged_start + r.length, device=dev)
    slots = bt[pos // cfg.block_size] * cfg.block_size + pos % cfg.block_size
    inv = 1.0 / (cfg.theta ** (torch.arange(0, cfg.head_size, 2, dtype=torch.float32)
                               / cfg.head_size))
    srcs = [wl.stores[0][li][r.store_start : r.store_start + r.length] for li in range(cfg.layers)]

    def turn():
        shift = ref_sk.rope_shift(r.delta, cfg.head_size, inv, dev)
        for src, kv in zip(srcs, wl.kv, strict=True):
            ref_sk.scatter_shifted(src, kv, slots, cfg.block_size, False, shift)

    ref_sk.warmup(wl.kv[0], cfg.block_size, False)
    for _ in range(max(warmup, 1)):
        turn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(steps):
        turn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    out = {"impl": "marathon.shift_kernels.scatter_shifted -> _shift_scatter_kernel "
                   "(reference Triton kernel, unmodified, baseline/_ref)",
           "value": round(cfg.algorithmic_bytes() / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
           "ms_per_turn": round(ms, 4), "launches_per_turn": cfg.layers,
           "device": torch.cuda.get_device_name(dev), "steps": steps,
           "note": "destination slots resident on the device; CUDA events around whole turns"}
    del wl, srcs
    torch.cuda.empty_cache()
    return out


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from marathon_b200.workloads import config

    cfg = config(args.config)
    cpu = CpuPath(cfg)
    t_layer, _ = cpu.run()
    # a step is one whole turn (every layer) unless K + W whole turns would take
    # more than about 150 s, in which case each step is a bounded run of layers
    budget = 150.0
    per_step = cfg.layers
    if (args.steps + args.warmup) * t_layer * cfg.layers > budget:
        per_step = max(1, int(budget / max((args.steps + args.warmup) * t_layer, 1e-9)))
    times, moved = [], 0
    for i in range(args.warmup + args.steps):
        dt, b = cpu.run(layers=per_step)
        if i >= args.warmup:
            times.append(dt)
            moved += b
    secs = sum(times)
    gbs = moved / secs / 1e9
    ms_step = secs / args.steps * 1e3
    whole = per_step == cfg.layers
    sample = (f"each step: one whole {cfg.name} turn ({cfg.layers} layers x {cpu.n} tokens)"
              if whole else f"each step: {per_step} of {cfg.layers} layers x {cpu.n} tokens")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3" if cfg.dtype == "e4m3" else "bf16", "data": "synthetic",
        "impl": "reference", "config": workload_config(cfg, world, args.layout),
        "ms_per_turn": round(ms_step * cfg.layers / per_step, 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu.threads,
                         "kind": cpu.kind, "impl": cpu.impl,
                         "sample": sample + f", torch CPU, {cpu.threads} threads"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if world == 1 and not args.no_triton and cpu.ref is not None and torch.cuda.is_available():
        try:
            line["reference_gpu"] = reference_triton(cfg, max(args.steps, 5), args.warmup)
        except Exception as e:  # noqa: BLE001 - report, never fail the CPU arm over it
            line["reference_gpu"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- native
def host_tier_timing(cfg, wl, args, names, jobs, fp8, turn_bytes, device) -> dict:
    """The same turn from a store in pinned host memory, through staged copies.

    Rows cross the host link once per step (copy engines into a device staging
    ring, ``mshift_stage``), then the ordinary load kernel runs from staging.
    The bound is the host-to-device copy bandwidth, measured here on one large
    pinned copy.
    """
    from marathon_b200.shift_store import ShiftStore
    from marathon_b200.worker import ShiftWorker

    # the link's own bandwidth: one 1 GiB pinned -> device copy, best of 3
    src = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    best = None
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        best = ms if best is None else min(best, ms)
    link = (1 << 30) / (best / 1e3) / 1e9
    del src, dst

    store = ShiftStore(budget_tokens=sum(cfg.history), device="cpu")
    for si, per_layer in enumerate(wl.stores):
        bufs = {}
        for n, t in zip(names, per_layer, strict=True):
            h = store.new_buffer(t.shape, t.dtype, "cpu")
            h.copy_(t)
            bufs[n] = h
        store.adopt(f"s{si}", bufs, 0, cfg.history[si])
    worker = ShiftWorker(store, cfg.block_size, wl.inv_freq.cpu(), layout=args.layout, fp8=fp8,
                         k_scales=wl.k_scales)
    worker.register(dict(zip(names, wl.kv, strict=True)))
    for _ in range(3):
        worker.load(jobs)
    steps = 5
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        worker.load(jobs, check=True)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    staged = worker.mover.last_staged_bytes
    # the asynchronous form a forward pass consumes layer by layer (host clock)
    issue, first, whole = [], [], []
    for _ in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        worker.load(jobs, asynchronous=True)
        issue.append(time.perf_counter() - t0)
        worker.pending.layer_done[0].synchronize()
        first.append(time.perf_counter() - t0)
        worker.finish_pending()
        whole.append(time.perf_counter() - t0)
    # the save direction: the same rows out of the paged caches into host memory
    from marathon_b200.worker import SaveJob

    saves = [SaveJob(j.session, j.src_start, j.length, block_ids=j.block_ids) for j in jobs]
    worker.save(saves)
    torch.cuda.synchronize()
    a.record()
    for _ in range(steps):
        worker.save(saves, check=True)
    b.record()
    torch.cuda.synchronize()
    save_ms = a.elapsed_time(b) / steps
    save_staged = worker.mover.last_staged_bytes
    return {
        "value": round(turn_bytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 3),
        "api": "marathon_b200.worker.ShiftWorker.load (store on device='cpu', pinned)",
        "save_ms_per_step": round(save_ms, 3),
        "save_link_achieved": round(save_staged / (save_ms / 1e3) / 1e9, 2),
        "staged_bytes_per_step": staged, "chunks": worker.mover.last_chunks,
        "copies": worker.mover.last_copies,
        "link_achieved": round(staged / (ms / 1e3) / 1e9, 2),
        "link_peak": round(link, 2), "link_frac": round(staged / (ms / 1e3) / 1e9 / link, 4),
        "link_peak_kind": "measured live: one 1 GiB pinned host->device copy",
        "steps": steps,
        "async": {"issue_ms": round(statistics.median(issue) * 1e3, 2),
                  "first_layer_ms": round(statistics.median(first) * 1e3, 2),
                  "all_layers_ms": round(statistics.median(whole) * 1e3, 2),
                  "clock": "host perf_counter, median of 3"},
    }


class Ranks:
    """This process's rank, the device and the group's barrier / max over ranks."""

    def __init__(self):
        import torch.distributed as dist

        self.dist = dist
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.device = torch.device("cuda", self.local)
        torch.cuda.set_device(self.device)
        if self.world > 1:
            dist.init_process_group("nccl", device_id=self.device,
                                    timeout=timedelta(seconds=180))

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(device_ids=[self.local])

    def max(self, x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, values: list[float]) -> list[list[float]]:
        """Every rank's ``values`` (same length on every rank), in rank order."""
        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        if self.world == 1:
            return [t.tolist()]
        out = [torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return [o.tolist() for o in out]

    def close(self):
        if self.world > 1:
            self.barrier()
            self.dist.destroy_process_group()


def load_step(launcher, wl, ev=None, check=False) -> tuple[int, int]:
    """One turn: pack + descriptor copy, table and load kernels; (launches, H2D bytes).

    The event pair brackets the table kernel and the load kernel together: an
    event between them would break the programmatic dependent launch that lets
    the load kernel's CTAs start while the table kernel ends.
    """
    p = launcher.prepare_load(wl.runs, wl.view, wl.inv_freq)
    if ev is not None:
        ev[0].record()
    n = launcher.launch(p)
    if ev is not None:
        ev[1].record()
    launcher.finish(p, check)
    return n, p.h2d_bytes


#: GPU cycles of the sleep queued ahead of a timed region (about 0.3 ms):
#: the stream stays busy while the host packs the region's first turn
LEAD_CYCLES = 600_000


def timed_turns(step, steps: int, ranks: Ranks, detail: dict | None = None):
    """``steps`` turns back to back, CUDA events around all of them (barrier and
    sync on both sides), max over ranks.

    No event sits between turns: one there ends the overlap of a load kernel
    with the next turn's table kernel (programmatic dependent launch), which
    measured on B200 costs a one-head turn 4-8 us; single-turn times come
    from ``isolated_turns`` after the region instead.  A GPU sleep of
    ``LEAD_CYCLES`` queued before the start event keeps the stream busy while
    the host packs the first turn, so the region holds no idle time from that
    packing.  Returns (max-over-ranks ms for all turns, launches); with
    ``detail``, also every rank's device ms and host (issuing) ms per turn."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    ranks.barrier()
    torch.cuda.synchronize()
    launches = 0
    torch.cuda._sleep(LEAD_CYCLES)
    t0 = time.perf_counter()
    start.record()
    for _ in range(steps):
        n, _ = step(None)
        launches += n
    end.record()
    host_ms = (time.perf_counter() - t0) * 1e3
    torch.cuda.synchronize()
    ranks.barrier()
    mine = start.elapsed_time(end)
    if detail is not None:
        rows = ranks.gather([mine / steps, host_ms / steps])
        detail.update({"ms_per_step": [round(r[0], 4) for r in rows],
                       "host_issue_ms_per_step": [round(r[1], 4) for r in rows]})
    return ranks.max(mine), launches


def isolated_turns(step, n: int, ranks: Ranks) -> dict:
    """``n`` turns each bracketed by its own CUDA events, after the timed region:
    the best and median single-turn time (max over ranks per turn).  Each turn
    starts cold (the event before it ends the programmatic overlap with the
    previous turn), so these are a little above the back-to-back mean."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n)]
    ranks.barrier()
    torch.cuda.synchronize()
    for pair in ev:
        step(pair)
    torch.cuda.synchronize()
    ms = [ranks.max(a.elapsed_time(b)) for a, b in ev]
    return {"n": n, "best_ms": round(min(ms), 4), "median_ms": round(statistics.median(ms), 4),
            "spans": "rope_tables_kernel + the load kernel, one turn at a time"}


def e2e_turns(worker, jobs, steps: int, ranks: Ranks) -> dict:
    """The turn through the public worker API from host metadata, back to back.

    Every step packs the descriptors and the block table on the host, copies
    them from pinned memory, runs the table and load kernels and copies the
    4-byte status word back; the status of a step is read on the host once
    the next step is queued, and the last one before the timed region closes.
    """
    for _ in range(3):
        worker.load(jobs)
    ranks.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        worker.load(jobs, asynchronous=True)  # checks the previous step's status
    worker.finish_pending()  # the last step's status, read on the host
    e1.record()
    torch.cuda.synchronize()
    ranks.barrier()
    return {"ms_per_step": ranks.max(e0.elapsed_time(e1)) / steps,
            "h2d_bytes_per_step": int(worker.launcher.last_h2d), "d2h_bytes_per_step": 4}


def worker_for(wl, cfg, layout, device, fp8):
    """A ShiftWorker over the workload's caches, its stores adopted as sessions."""
    from marathon_b200.shift_store import ShiftStore
    from marathon_b200.worker import LoadJob, ShiftWorker

    names = [f"layer.{i}" for i in range(cfg.layers)]
    store = ShiftStore(budget_tokens=sum(cfg.history), device=str(device))
    for si, per_layer in enumerate(wl.stores):
        store.adopt(f"s{si}", dict(zip(names, per_layer, strict=True)), 0, cfg.history[si])
    worker = ShiftWorker(store, cfg.block_size, wl.inv_freq.cpu(), layout=layout, fp8=fp8,
                         k_scales=wl.k_scales)
    worker.register(dict(zip(names, wl.kv, strict=True)))
    jobs = [LoadJob(f"s{si}", s.src_start, s.delta, s.dst_start, s.length,
                    block_ids=wl.block_tables_host[si])
            for si, segs in enumerate(cfg.segments) for s in segs]
    return worker, jobs, names


def roofline(rank_bytes: int, launch_ms: float, traffic, kernel: str) -> dict:
    """The load kernel against the HBM roofline.

    ``launch_ms`` is the kernel's average launch duration over the timed
    region: the region's device time (CUDA events, max over ranks) over the
    load launches in it, one per turn, back to back; the turn's table kernel
    (about 3-5 us) overlaps the previous load through programmatic dependent
    launch, and the ncu launch list gives the load kernel 99.7% of a turn's
    kernel time.
    """
    peak, peak_kind = peaks()
    achieved = rank_bytes / (launch_ms / 1e3) / 1e9
    return {
        "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
        "frac_of_8tbs": round(achieved / 8000.0, 4), "kernel": kernel,
        "kernel_ms": round(launch_ms, 4),
        "kernel_ms_spans": "timed region device time (max over ranks) / load launches in it; "
                           "launches back to back, the table kernel overlapping",
        "bytes_per_launch": rank_bytes,
        "traffic": round(traffic) if traffic else None,
    }


def fp8_torch_check(wl) -> dict:
    """Every layer of an e4m3 turn against a torch restatement on the GPU of
    dequantise -> rotate -> requantise (fp32, the reference's tables as its GPU
    path builds them, separate multiply and add kernels, divide by the layer's
    K scale, saturate to +-448, round to e4m3): V bit-exact, K within one step."""
    d = wl.cfg.head_size
    worst = differ = total = 0
    v_exact = True
    for r in wl.runs:
        bt = r.block_table.long()
        pos = torch.arange(r.paged_start, r.paged_start + r.length, device=bt.device)
        blk, off = bt[pos // wl.cfg.block_size], pos % wl.cfg.block_size
        ang = float(r.delta) * wl.inv_freq
        cos, sin = torch.cat((ang, ang)).cos(), torch.cat((ang, ang)).sin()
        for li in range(wl.cfg.layers):
            rows = wl.stores[r.session][li][r.store_start : r.store_start + r.length]
            got = wl.kv[li][blk, off]
            ks = wl.k_scales[li]
            kf = rows[..., :d].float() * ks
            turned = torch.cat((-kf[..., d // 2 :], kf[..., : d // 2]), dim=-1)
            want = ((kf * cos + turned * sin) / ks).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)

            def order(t):
                u = t.view(torch.uint8).int()
                return torch.where(u >= 128, 128 - u, u)

            steps = (order(got[..., :d]) - order(want)).abs()
            worst = max(worst, int(steps.max()))
            differ += int((steps > 0).sum())
            total += steps.numel()
            v_exact &= bool(torch.equal(got[..., d:].view(torch.uint8),
                                        rows[..., d:].view(torch.uint8)))
    return {"k_max_steps": worst, "k_codes_one_step_off": differ, "k_codes": total,
            "v_bit_exact": v_exact,
            "reference": "torch fp32 dequantise -> rotate -> divide -> saturate -> e4m3 on "
                         "the GPU, every layer"}


def c3_extra(args, ranks: Ranks) -> dict:
    """The FP8 turn (c3) on one GPU: the load kernel, the end-to-end call, the check."""
    from marathon_b200.paged import KVLayers
    from marathon_b200.shift_kernels import Launcher, set_load_kernel
    from marathon_b200.workloads import build, config

    cfg = config("c3")
    wl = build(cfg, ranks.device, layout=args.layout)
    wl.view = wl.store_view()
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, args.layout, fp8=True),
                        staging_slots=BENCH_SLOTS)
    load_step(launcher, wl, check=True)
    for _ in range(args.warmup):
        load_step(launcher, wl)
    steps = max(args.steps, 10)
    total_ms, _ = timed_turns(lambda ev: load_step(launcher, wl, ev), steps, ranks)
    ms = total_ms / steps
    out = {"config": workload_config(cfg, 1, args.layout), "metric": METRIC,
           "value": round(cfg.algorithmic_bytes() / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
           "ms_per_step": round(ms, 4), "steps": steps, "target_ms": 0.781,
           "roofline": roofline(wl.algorithmic_bytes(), ms,
                                traffic_for(cfg.name, args.layout,
                                            cfg.shifted_tokens * cfg.layers),
                                "bulk_load_kernel (mshift_load, TMA)")}
    prev = set_load_kernel("lsu")
    try:
        lsu_total, _ = timed_turns(lambda ev: load_step(launcher, wl, ev), 10, ranks)
    finally:
        set_load_kernel(prev)
    lsu_ms = lsu_total / 10
    out["roofline"]["alternatives"] = {"lsu": {
        "kernel": "move_kernel<load> (128-bit loads)", "kernel_ms": round(lsu_ms, 4),
        "achieved": round(wl.algorithmic_bytes() / (lsu_ms / 1e3) / 1e9, 1)}}
    worker, jobs, _ = worker_for(wl, cfg, args.layout, ranks.device, True)
    e = e2e_turns(worker, jobs, max(10, min(args.steps, 100)), ranks)
    out["e2e"] = {"value": round(cfg.algorithmic_bytes() / (e["ms_per_step"] / 1e3) / 1e9, 2),
                  "unit": "GB/s", "ms_per_step": round(e["ms_per_step"], 4),
                  "h2d_bytes_per_step": e["h2d_bytes_per_step"],
                  "d2h_bytes_per_step": e["d2h_bytes_per_step"],
                  "api": "marathon_b200.worker.ShiftWorker.load"}
    load_step(launcher, wl, check=True)
    torch.cuda.synchronize()
    out["check"] = fp8_torch_check(wl)
    del worker, jobs, launcher, wl
    torch.cuda.empty_cache()
    return out


def c4_extra(args, ranks: Ranks) -> dict:
    """64 sessions (c4) in one launch per rank at TP ``world``, each rank its head shard."""
    from marathon_b200.paged import KVLayers
    from marathon_b200.sharding import head_shard
    from marathon_b200.shift_kernels import Launcher
    from marathon_b200.workloads import build, config

    cfg = config("c4")
    lo, hi = head_shard(cfg.heads, ranks.rank, ranks.world)
    # store rows of every session plus a paged cache of about the same size
    need = sum(cfg.history) * cfg.layers * cfg.bytes_per_token_layer(hi - lo)
    free, _ = torch.cuda.mem_get_info(ranks.device)
    if ranks.max(float(need + (4 << 30) > free)) > 0:  # one decision for every rank
        return {"config": workload_config(cfg, ranks.world, args.layout),
                "skipped": f"needs about {need / 1e9:.0f} GB per GPU at {hi - lo} heads"}
    wl = build(cfg, ranks.device, head_lo=lo, head_hi=hi, layout=args.layout)
    wl.view = wl.store_view()
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, args.layout),
                        staging_slots=BENCH_SLOTS)
    load_step(launcher, wl, check=True)
    for _ in range(args.warmup):
        load_step(launcher, wl)
    steps = max(args.steps, 10)
    total_ms, _ = timed_turns(lambda ev: load_step(launcher, wl, ev), steps, ranks)
    ms = total_ms / steps
    out = {"config": workload_config(cfg, ranks.world, args.layout), "metric": METRIC,
           "value": round(cfg.algorithmic_bytes() / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
           "ms_per_step": round(ms, 4), "steps": steps, "runs": len(wl.runs),
           "roofline": roofline(wl.algorithmic_bytes(), ms, None,
                                "move_kernel<load> (mshift_load)")}
    worker, jobs, _ = worker_for(wl, cfg, args.layout, ranks.device, False)
    e = e2e_turns(worker, jobs, max(10, min(args.steps, 50)), ranks)
    out["e2e"] = {"value": round(cfg.algorithmic_bytes() / (e["ms_per_step"] / 1e3) / 1e9, 2),
                  "unit": "GB/s", "ms_per_step": round(e["ms_per_step"], 4),
                  "h2d_bytes_per_step": e["h2d_bytes_per_step"],
                  "d2h_bytes_per_step": e["d2h_bytes_per_step"],
                  "api": "marathon_b200.worker.ShiftWorker.load"}
    del worker, jobs, launcher, wl
    torch.cuda.empty_cache()
    return out


def native_arm(args) -> None:
    from marathon_b200.paged import KVLayers
    from marathon_b200.sharding import broadcast_table, head_shard, pack_table
    from marathon_b200.shift_kernels import Launcher, RunSpec
    from marathon_b200.workloads import build, config, scaled

    ranks = Ranks()
    device, rank, world = ranks.device, ranks.rank, ranks.world
    cfg = config(args.config)
    if args.layers:
        cfg = scaled(cfg, args.layers)
    share = args.rank_share if world == 1 and args.rank_share > 1 else 0
    h_lo, h_hi = head_shard(cfg.heads, 0, share) if share else head_shard(cfg.heads, rank, world)
    # store rows of every session plus a paged cache of about the same size,
    # per rank (bytes_per_token_layer counts a row twice: read and write)
    need = sum(cfg.history) * cfg.layers * cfg.bytes_per_token_layer(h_hi - h_lo)
    _, total = torch.cuda.mem_get_info(device)
    if need > total:
        raise SystemExit(f"{cfg.name} needs about {need / 1e9:.0f} GB per GPU at "
                         f"{h_hi - h_lo} heads per rank, more than the GPU's "
                         f"{total / 1e9:.0f} GB (run it over more GPUs)")
    wl = build(cfg, device, head_lo=h_lo, head_hi=h_hi, layout=args.layout)
    wl.view = wl.store_view()
    fp8 = cfg.dtype == "e4m3"
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, args.layout, fp8=fp8),
                        tile_tokens=args.tile_tokens or None, staging_slots=BENCH_SLOTS)

    # control plane: the segment table is rank 0's, broadcast once over NCCL
    if world > 1:
        mine = pack_table(wl.runs)
        got = broadcast_table(mine if rank == 0 else None, len(wl.runs), device=device)
        if not torch.equal(mine, got.cpu()):
            raise SystemExit(f"rank {rank}: segment table differs from rank 0's")

    def step(ev=None):
        return load_step(launcher, wl, ev)

    load_step(launcher, wl, check=True)  # first call: surface any rejected token before timing
    clocks = Clocks(device)
    clocks.start()
    t_warm = time.perf_counter()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # keep the GPU busy until nvidia-smi (slow to start) has sampled under load
    while time.perf_counter() - t_warm < 1.5:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    per_rank: dict = {}
    max_ms, launches = timed_turns(step, args.steps, ranks, per_rank)
    clk = clocks.stop()
    rank_bytes = wl.algorithmic_bytes()
    # the whole turn, all heads, all ranks (with --rank-share: that share only)
    turn_bytes = rank_bytes if share else cfg.algorithmic_bytes()
    ms_per_step = max_ms / args.steps
    value = turn_bytes / (ms_per_step / 1e3) / 1e9
    isolated = isolated_turns(step, 10, ranks)

    # the alternative load kernel (TMA bulk copies), kernel alone, same turn
    alt = None
    if not args.no_alt:
        from marathon_b200.shift_kernels import set_load_kernel

        prev = set_load_kernel("lsu" if fp8 else "bulk")  # the one auto did not pick
        try:
            load_step(launcher, wl, check=True)
            n_alt = max(10, min(args.steps, 100))
            a_total, _ = timed_turns(step, n_alt, ranks)
            name = ("lsu", "move_kernel<load> (128-bit loads)") if fp8 else (
                "bulk", "bulk_load_kernel (TMA cp.async.bulk, mbarrier ring)")
            m = a_total / n_alt
            alt = {name[0]: {"kernel": name[1], "kernel_ms": round(m, 4),
                             "achieved": round(rank_bytes / (m / 1e3) / 1e9, 1)}}
        finally:
            set_load_kernel(prev)

    # the save kernel on the same turn: paged rows of each run back to its store rows
    save = None
    if not args.no_save:
        sruns = [RunSpec(r.session, r.store_start, r.length, block_table=r.block_table,
                         paged_start=r.paged_start) for r in wl.runs]
        sp = launcher.prepare_save(sruns, wl.view)
        launcher.launch(sp)
        launcher.finish(sp, True)
        sev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(max(10, min(args.steps, 100)))]
        for a, b in sev:
            sp = launcher.prepare_save(sruns, wl.view)
            a.record()
            launcher.launch(sp)
            b.record()
            launcher.finish(sp, False)
        torch.cuda.synchronize()
        s_ms = statistics.mean(a.elapsed_time(b) for a, b in sev)
        save = {"kernel": "move_kernel<save> (mshift_save)", "kernel_ms": round(s_ms, 4),
                "achieved": round(rank_bytes / (s_ms / 1e3) / 1e9, 1)}

    # end to end through the public worker API, from host metadata
    e2e = None
    host_tier = None
    if not args.no_e2e:
        worker, jobs, names = worker_for(wl, cfg, args.layout, device, fp8)
        e = e2e_turns(worker, jobs, max(10, min(args.steps, 100)), ranks)
        e2e = {"value": round(turn_bytes / (e["ms_per_step"] / 1e3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(e["ms_per_step"], 4),
               "h2d_bytes_per_step": e["h2d_bytes_per_step"],
               "d2h_bytes_per_step": e["d2h_bytes_per_step"],
               "api": "marathon_b200.worker.ShiftWorker.load",
               "status_read": "each step's 4-byte status is copied back every step and read "
                              "on the host once the next step is queued; the last inside "
                              "the timed region"}
        if world == 1 and not share and not args.no_host_tier:
            host_tier = host_tier_timing(cfg, wl, args, names, jobs, fp8, turn_bytes, device)
        del worker, jobs

    units = cfg.shifted_tokens * cfg.layers  # (token, layer) units of the whole turn
    traffic = traffic_for(cfg.name, args.layout, units)
    if traffic is not None:
        traffic *= (h_hi - h_lo) / cfg.heads  # this rank's head shard of each unit
    roof = roofline(rank_bytes, ms_per_step, traffic,
                    "bulk_load_kernel (mshift_load, TMA)" if fp8
                    else "move_kernel<load> (mshift_load)")
    roof["alternatives"] = alt
    roof["isolated_turns"] = isolated
    cpu = None
    if rank == 0 and world == 1 and not share and not args.no_cpu_baseline:
        base = CpuPath(cfg)
        smp = base.sample(args.cpu_seconds)
        cpu = {"value": round(smp["gbs"], 3), "unit": "GB/s", "cores": base.threads,
               "kind": base.kind, "impl": base.impl, "sample": smp["sample"],
               "ms_per_turn_extrapolated": round(smp["ms_per_layer"] * cfg.layers, 1)}
        del base
    tile_tokens = launcher.tile_tokens
    del launcher, wl
    torch.cuda.empty_cache()

    extra = {}
    if not args.no_extra and args.config == "c2" and not args.layers and not share:
        if world == 1:
            extra["c3"] = c3_extra(args, ranks)
        else:
            extra["c4"] = c4_extra(args, ranks)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "e4m3" if fp8 else "bf16",
            "data": "synthetic",
            "config": workload_config(cfg, world, args.layout, share),
            "gib_s": round(turn_bytes / (ms_per_step / 1e3) / 2**30, 2),
            "launch": {"tile_tokens": tile_tokens},
            "roofline": roof,
            "e2e": e2e,
            "save": save,
            "host_tier": host_tier,
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clk,
            "per_rank": per_rank if world > 1 else None,
            **extra,
        }
        print(json.dumps(line), flush=True)
    ranks.close()


def main() -> None:
    args = parse()
    sys.path.insert(0, str(ROOT))
    if args.impl == "reference":
        reference_arm(args)
    else:
        native_arm(args)


if __name__ == "__main__":
    main()
