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
  roofline      load kernel alone: algorithmic bytes per launch / mean CUDA-event
                duration of that launch, against the measured HBM copy peak
  e2e           the same turn through the public worker API (ShiftWorker.load)
                from host metadata: block table + descriptors copied from pinned
                host memory, tables + load kernels, the 4-byte status read back
  cpu_baseline  the reference's torch CPU path on this host, bounded sample
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
    ap.add_argument("--no-save", action="store_true", help="skip the save-kernel timing")
    ap.add_argument("--no-alt", action="store_true", help="skip the TMA bulk-load timing")
    ap.add_argument("--no-host-tier", action="store_true",
                    help="skip the pinned-host store tier timing (N=1 only)")
    return ap.parse_args()


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
class CpuPath:
    """The reference's torch CPU path on two resident layers of ``cfg``'s first segment."""

    def __init__(self, cfg):
        from oracle import shift_oracle as O
        from oracle import torch_cpu_path as T

        self.T = T
        self.cfg = cfg
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        seg = cfg.segments[0][0]
        self.n, h, d, bs = seg.length, cfg.heads, cfg.head_size, cfg.block_size
        blocks = -(-seg.dst_end // bs) + 16
        table = np.random.default_rng(0).permutation(blocks).astype(np.int64)
        self.slots = torch.from_numpy(O.slots(table, seg.dst_start, seg.dst_end, bs))
        inv = O.inv_freq(d, cfg.theta)
        self.emb = T.emb_tables(torch.from_numpy(O.rope_tables([seg.delta], inv)[0]))
        g = torch.Generator().manual_seed(0)
        self.fp8 = cfg.dtype == "e4m3"
        if self.fp8:  # codes of the c3 distribution: values / per-layer scale, saturated
            self.k_scale = 0.05
            self.srcs = [(torch.randn(self.n, h, 2 * d, generator=g) * 20).clamp(-448, 448)
                         .to(torch.float8_e4m3fn) for _ in range(2)]
            self.kvs = [torch.zeros(blocks, bs, h, 2 * d, dtype=torch.float8_e4m3fn)
                        for _ in range(2)]
        else:
            self.srcs = [torch.randn(self.n, h, 2 * d, generator=g).to(torch.bfloat16)
                         for _ in range(2)]
            self.kvs = [torch.zeros(blocks, bs, h, 2 * d, dtype=torch.bfloat16) for _ in range(2)]
        self.bs = bs
        self.i = 0
        self.run(tokens=256)  # first touch

    def run(self, tokens: int | None = None) -> tuple[float, int]:
        """One layer (or its first ``tokens`` tokens); returns (seconds, bytes moved)."""
        n = self.n if tokens is None else min(tokens, self.n)
        k = self.i % 2
        self.i += 1
        t0 = time.perf_counter()
        if self.fp8:
            self.T.scatter_layer_e4m3(self.srcs[k][:n], self.kvs[k], self.slots[:n], self.bs,
                                      False, self.emb, self.k_scale)
        else:
            self.T.scatter_layer(self.srcs[k][:n], self.kvs[k], self.slots[:n], self.bs, False,
                                 self.emb)
        return time.perf_counter() - t0, n * self.cfg.bytes_per_token_layer()

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
                          f"{self.cfg.dtype} each, torch CPU, {self.threads} threads"}


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from marathon_b200.workloads import config

    cfg = config(args.config)
    seg = cfg.segments[0][0]
    cpu = CpuPath(cfg)
    t_layer, _ = cpu.run()
    # each step is a bounded slice of one layer so K + W steps fit in about two minutes
    budget = 120.0 / max(args.steps + args.warmup, 1)
    tokens = max(256, min(seg.length, int(seg.length * budget / max(t_layer, 1e-6))))
    secs = moved = 0.0
    for i in range(args.warmup + args.steps):
        dt, b = cpu.run(tokens)
        if i >= args.warmup:
            secs += dt
            moved += b
    gbs = moved / secs / 1e9
    ms_turn = cfg.algorithmic_bytes() / (gbs * 1e9) * 1e3
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_turn, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": cfg.dtype, "data": "synthetic", "impl": "reference",
        "config": {"workload": f"{cfg.name} {cfg.model} shift turn", "layers": cfg.layers,
                   "tokens_shifted": seg.length, "delta": seg.delta, "heads": cfg.heads,
                   "head_size": cfg.head_size, "block_size": cfg.block_size, "layout": "nhd",
                   "turn_bytes": cfg.algorithmic_bytes()},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu.threads,
                         "kind": "port",
                         "sample": f"each step: {tokens} of {seg.length} tokens of one layer "
                                   "(torch CPU path); ms_per_step extrapolates to the "
                                   f"{cfg.layers}-layer turn"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
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


def native_arm(args) -> None:
    import torch.distributed as dist

    from marathon_b200.paged import KVLayers
    from marathon_b200.sharding import broadcast_table, head_shard, pack_table
    from marathon_b200.shift_kernels import Launcher
    from marathon_b200.shift_store import ShiftStore
    from marathon_b200.worker import LoadJob, ShiftWorker
    from marathon_b200.shift_kernels import RunSpec
    from marathon_b200.workloads import build, config, scaled

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=180))

    cfg = config(args.config)
    if args.layers:
        cfg = scaled(cfg, args.layers)
    h_lo, h_hi = head_shard(cfg.heads, rank, world)
    # store rows of every session plus a paged cache of about the same size,
    # per rank (bytes_per_token_layer counts a row twice: read and write)
    need = sum(cfg.history) * cfg.layers * cfg.bytes_per_token_layer(h_hi - h_lo)
    _, total = torch.cuda.mem_get_info(device)
    if need > total:
        raise SystemExit(f"{cfg.name} needs about {need / 1e9:.0f} GB per GPU at "
                         f"{h_hi - h_lo} heads per rank, more than the GPU's "
                         f"{total / 1e9:.0f} GB (run it over more GPUs)")
    wl = build(cfg, device, head_lo=h_lo, head_hi=h_hi, layout=args.layout)
    fp8 = cfg.dtype == "e4m3"
    layers = KVLayers(wl.kv, cfg.block_size, args.layout, fp8=fp8)
    launcher = Launcher(layers, tile_tokens=args.tile_tokens or None)
    view = wl.store_view()

    # control plane: the segment table is rank 0's, broadcast once over NCCL
    if world > 1:
        mine = pack_table(wl.runs)
        got = broadcast_table(mine if rank == 0 else None, len(wl.runs), device=device)
        if not torch.equal(mine, got.cpu()):
            raise SystemExit(f"rank {rank}: segment table differs from rank 0's")

    def step(check=False, ev=None):
        # the event pair brackets the table kernel and the load kernel together:
        # an event between them would break the programmatic dependent launch
        # that lets the load kernel's CTAs start while the table kernel ends
        p = launcher.prepare_load(wl.runs, view, wl.inv_freq, k_scales=wl.k_scales)
        if ev is not None:
            ev[0].record()
        n = launcher.launch(p)
        if ev is not None:
            ev[1].record()
        launcher.finish(p, check)
        return n, p.h2d_bytes

    step(check=True)  # first call: surface any rejected token before timing
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

    # kernel durations are sampled on every `stride`-th step (at least 25
    # samples): a timing-event pair costs the step a few microseconds, which
    # per-step sampling would charge to every step of the whole-job number
    stride = max(1, args.steps // 25)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(0, args.steps, stride)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    launches = 0
    start.record()
    for i in range(args.steps):
        n, _ = step(ev=kev[i // stride] if i % stride == 0 else None)
        launches += n
    end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier(device_ids=[local])
    elapsed = start.elapsed_time(end)
    per_step = [a.elapsed_time(b) for a, b in kev]
    kernel_ms = statistics.mean(per_step)
    t = torch.tensor([elapsed], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    turn_bytes = cfg.algorithmic_bytes()  # the whole turn, all heads, all ranks
    rank_bytes = wl.algorithmic_bytes()
    ms_per_step = max_ms / args.steps
    value = turn_bytes / (ms_per_step / 1e3) / 1e9

    # the alternative load kernel (TMA bulk copies), kernel alone, same turn
    alt = None
    if not args.no_alt:
        from marathon_b200.shift_kernels import set_load_kernel

        prev = set_load_kernel("lsu" if fp8 else "bulk")  # the one auto did not pick
        try:
            aev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(max(10, min(args.steps, 100)))]
            step(check=True)
            for a_, b_ in aev:
                step(ev=(a_, b_))
            torch.cuda.synchronize()
            a_ms = statistics.mean(a_.elapsed_time(b_) for a_, b_ in aev)
            name = ("lsu", "move_kernel<load> (128-bit loads)") if fp8 else (
                "bulk", "bulk_load_kernel (TMA cp.async.bulk, mbarrier ring)")
            alt = {name[0]: {"kernel": name[1], "kernel_ms": round(a_ms, 4),
                             "achieved": round(rank_bytes / (a_ms / 1e3) / 1e9, 1)}}
        finally:
            set_load_kernel(prev)

    # the save kernel on the same turn: paged rows of each run back to its store rows
    save = None
    if not args.no_save:
        sruns = [RunSpec(r.session, r.store_start, r.length, block_table=r.block_table,
                         paged_start=r.paged_start) for r in wl.runs]
        sp = launcher.prepare_save(sruns, view)
        launcher.launch(sp)
        launcher.finish(sp, True)
        sev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(max(10, min(args.steps, 100)))]
        for a, b in sev:
            sp = launcher.prepare_save(sruns, view)
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
    if not args.no_e2e:
        names = [f"layer.{i}" for i in range(cfg.layers)]
        store = ShiftStore(budget_tokens=sum(cfg.history), device=str(device))
        for si, per_layer in enumerate(wl.stores):
            store.adopt(f"s{si}", dict(zip(names, per_layer, strict=True)), 0, cfg.history[si])
        worker = ShiftWorker(store, cfg.block_size, wl.inv_freq.cpu(), layout=args.layout,
                             fp8=fp8, k_scales=wl.k_scales)
        worker.register(dict(zip(names, wl.kv, strict=True)))
        jobs = [LoadJob(f"s{si}", s.src_start, s.delta, s.dst_start, s.length,
                        block_ids=wl.block_tables_host[si])
                for si, segs in enumerate(cfg.segments) for s in segs]
        for _ in range(3):
            worker.load(jobs)
        e_steps = max(10, min(args.steps, 100))
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        h2d = 0
        for _ in range(e_steps):
            worker.load(jobs, check=True)  # packs, copies, launches, reads the status back
            h2d = worker.launcher.last_h2d
        e1.record()
        torch.cuda.synchronize()
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e_ms = float(et.item()) / e_steps
        e2e = {"value": round(turn_bytes / (e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(e_ms, 4), "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": 4, "api": "marathon_b200.worker.ShiftWorker.load"}

    host_tier = None
    if world == 1 and not args.no_host_tier and not args.no_e2e:
        host_tier = host_tier_timing(cfg, wl, args, names, jobs, fp8, turn_bytes, device)

    peak, peak_kind = peaks()
    achieved = rank_bytes / (kernel_ms / 1e3) / 1e9
    units = cfg.shifted_tokens * cfg.layers  # (token, layer) units of the whole turn
    traffic = traffic_for(cfg.name, args.layout, units)
    if traffic is not None:
        traffic *= (h_hi - h_lo) / cfg.heads  # this rank's head shard of each unit
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        s = CpuPath(cfg).sample(args.cpu_seconds)
        cpu = {"value": round(s["gbs"], 3), "unit": "GB/s", "cores": os.cpu_count() or 1,
               "kind": "port", "sample": s["sample"],
               "ms_per_turn_extrapolated": round(s["ms_per_layer"] * cfg.layers, 1)}

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
            "config": {
                "workload": f"{cfg.name} {cfg.model} shift turn",
                "layers": cfg.layers, "tokens_shifted": cfg.shifted_tokens,
                "deltas": sorted({s.delta for segs in cfg.segments for s in segs}),
                "heads": cfg.heads, "heads_per_rank": h_hi - h_lo, "head_size": cfg.head_size,
                "block_size": cfg.block_size, "layout": args.layout, "parallelism":
                f"kv-head shard tp{world}", "turn_bytes": turn_bytes,
                "gib_s": round(turn_bytes / (ms_per_step / 1e3) / 2**30, 2),
                "l2": "inputs larger than L2 (store + paged cache per step >> 126 MB)",
                "tile_tokens": launcher.tile_tokens,
            },
            "roofline": {
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "frac_of_8tbs": round(achieved / 8000.0, 4),
                "kernel": ("bulk_load_kernel (mshift_load, TMA)" if fp8
                           else "move_kernel<load> (mshift_load)"),
                "kernel_ms": round(kernel_ms, 4),
                "kernel_ms_spans": "rope_tables_kernel + the load kernel (one event pair "
                                   "around both; the table kernel is ~0.3% of a c2 step)",
                "kernel_samples": len(per_step),
                "kernel_ms_best": round(min(per_step), 4),
                "kernel_ms_median": round(statistics.median(per_step), 4),
                "bytes_per_launch": rank_bytes,
                "traffic": round(traffic) if traffic else None,
                "alternatives": alt,
            },
            "e2e": e2e,
            "save": save,
            "host_tier": host_tier,
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main() -> None:
    args = parse()
    sys.path.insert(0, str(ROOT))
    if args.impl == "reference":
        reference_arm(args)
    else:
        native_arm(args)


if __name__ == "__main__":
    main()
