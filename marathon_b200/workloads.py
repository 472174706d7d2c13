"""Seeded synthetic shift turns with the shapes of the benchmark configurations c0-c4.

The reference benchmarks only synthetic shapes (``scripts/bench_shift_copy.py``
builds random stores and a ``randperm`` block table); these are the same kind
of inputs at the five configurations the build is measured on:

c0  Qwen3-0.6B: 28 layers, 4,096 cached tokens, one segment [1024, 4096) -> +37,
    destination table a seeded permutation of 300 free blocks
c1  Qwen3-8B: 36 layers, 16,384 tokens, three segments at +12 / -40 / +215 with
    seeded, non-block-aligned boundaries
c2  Qwen3-14B: 40 layers, 30,720 tokens, an edit at 2048 replacing 64 tokens by
    244: [2112, 30720) -> +180, 28,608 tokens
c3  c2 in float8_e4m3fn with per-layer scales ~ U(0.01, 0.1)
c4  64 Qwen3-8B sessions, history ~ U[2k, 32k], 1-8 segments, delta ~ U[-512, 512]

All share 8 KV heads, head_size 128, block 16, NeoX RoPE with theta 1e6.  K
and V are N(0, 1) times a per-(layer, head, channel) scale drawn log-uniform in
[0.1, 10].  A rank of a head-sharded run holds heads ``[head_lo, head_hi)``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .shift_kernels import RunSpec, StoreView, inv_freq

HEADS, HEAD_SIZE, BLOCK, THETA = 8, 128, 16, 1e6


@dataclass(frozen=True)
class Segment:
    """``length`` tokens moving from store position ``src_start`` to ``dst_start``."""

    src_start: int
    dst_start: int
    length: int

    @property
    def delta(self) -> int:
        return self.dst_start - self.src_start

    @property
    def dst_end(self) -> int:
        return self.dst_start + self.length


@dataclass(frozen=True)
class Config:
    name: str
    model: str
    layers: int
    history: tuple[int, ...]  # cached tokens of each session (store capacity)
    segments: tuple[tuple[Segment, ...], ...]  # per session
    dtype: str = "bf16"
    heads: int = HEADS
    head_size: int = HEAD_SIZE
    block_size: int = BLOCK
    theta: float = THETA
    free_blocks: tuple[int, ...] = ()  # destination blocks reserved per session (0 = tight)

    @property
    def sessions(self) -> int:
        return len(self.history)

    @property
    def shifted_tokens(self) -> int:
        return sum(s.length for segs in self.segments for s in segs)

    def bytes_per_token_layer(self, heads: int | None = None) -> int:
        """Algorithmic bytes of one shifted (token, layer): read + write of 2*H*D elements."""
        es = 1 if self.dtype == "e4m3" else 2
        h = self.heads if heads is None else heads
        return 2 * 2 * h * self.head_size * es

    def algorithmic_bytes(self, heads: int | None = None) -> int:
        return self.shifted_tokens * self.layers * self.bytes_per_token_layer(heads)


def _c1_segments(seed: int = 1) -> tuple[Segment, ...]:
    rng = np.random.default_rng(seed)

    def unaligned(lo, hi):
        while True:
            v = int(rng.integers(lo, hi))
            if v % BLOCK:
                return v

    b0, b1 = unaligned(4000, 6000), unaligned(10000, 12000)
    return (
        Segment(0, 12, b0),
        Segment(b0 + 60, b0 + 20, b1 - b0 - 60),
        Segment(b1, b1 + 215, 16384 - b1),
    )


def c4_config(seed: int = 4, sessions: int = 64) -> Config:
    """64 sessions with seeded histories and 1-8 non-overlapping segments each."""
    rng = np.random.default_rng(seed)
    hist, segs = [], []
    for _ in range(sessions):
        h = int(rng.integers(2048, 32769))
        k = int(rng.integers(1, 9))
        cuts = np.sort(rng.choice(np.arange(64, h - 64), size=2 * k, replace=False))
        mine, floor = [], 0
        for j in range(k):
            a, b = int(cuts[2 * j]), int(cuts[2 * j + 1])
            d = int(rng.integers(-512, 513))
            dst = max(a + d, floor)
            mine.append(Segment(a, dst, b - a))
            floor = dst + (b - a)
        hist.append(h)
        segs.append(tuple(mine))
    return Config("c4", "Qwen3-8B x64", 36, tuple(hist), tuple(segs))


CONFIGS: dict[str, Config] = {
    "c0": Config("c0", "Qwen3-0.6B", 28, (4096,), ((Segment(1024, 1061, 3072),),),
                 free_blocks=(300,)),
    # c0 with the prefix moved too, as a delta-0 segment (a plain paged copy)
    "c0z": Config("c0z", "Qwen3-0.6B", 28, (4096,),
                  ((Segment(0, 0, 1024), Segment(1024, 1061, 3072)),), free_blocks=(300,)),
    "c1": Config("c1", "Qwen3-8B", 36, (16384,), (_c1_segments(),)),
    "c2": Config("c2", "Qwen3-14B", 40, (30720,), ((Segment(2112, 2292, 28608),),)),
    "c3": Config("c3", "Qwen3-14B", 40, (30720,), ((Segment(2112, 2292, 28608),),),
                 dtype="e4m3"),
}


def config(name: str) -> Config:
    if name == "c4":
        return c4_config()
    return CONFIGS[name]


def scaled(cfg: Config, layers: int | None = None) -> Config:
    """The same turn with fewer layers (for oracle-sized parity checks)."""
    return Config(cfg.name, cfg.model, layers or cfg.layers, cfg.history, cfg.segments,
                  cfg.dtype, cfg.heads, cfg.head_size, cfg.block_size, cfg.theta, cfg.free_blocks)


@dataclass
class Workload:
    """Device-resident inputs of one shift turn (one rank's head shard)."""

    cfg: Config
    head_lo: int
    head_hi: int
    stores: list[list[torch.Tensor]]  # [session][layer] -> [cap, h, 2D]
    kv: list[torch.Tensor]  # [layer] paged cache (layout per `layout`)
    layout: str
    block_tables: list[torch.Tensor]  # [session] int32 device
    block_tables_host: list[np.ndarray]
    runs: list[RunSpec]
    inv_freq: torch.Tensor
    k_scales: torch.Tensor | None
    v_scales: torch.Tensor | None
    keep: list = field(default_factory=list)

    @property
    def heads(self) -> int:
        return self.head_hi - self.head_lo

    def store_view(self) -> StoreView:
        S, L = len(self.stores), len(self.kv)
        ptrs = np.zeros((S, L), dtype=np.uint64)
        caps = np.zeros(S, dtype=np.int64)
        for s in range(S):
            caps[s] = self.stores[s][0].shape[0]
            for li in range(L):
                ptrs[s, li] = self.stores[s][li].data_ptr()
        t = self.stores[0][0]
        return StoreView(ptrs, caps, t.stride(0), t.stride(1))

    def algorithmic_bytes(self) -> int:
        return self.cfg.algorithmic_bytes(self.heads)


def _channel_scales(cfg: Config, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    lo, hi = math.log(0.1), math.log(10.0)
    u = torch.rand(cfg.layers, cfg.heads, 2 * cfg.head_size, generator=g)
    return torch.exp(lo + (hi - lo) * u)


def _paged_shape(layout: str, blocks: int, bs: int, h: int, d: int):
    if layout == "nhd":
        return (blocks, bs, h, 2 * d)
    if layout == "hnd":
        return (blocks, h, bs, 2 * d)
    if layout == "split":
        return (2, blocks, bs, h, d)
    if layout == "split_blocks":
        return (blocks, 2, bs, h, d)
    raise ValueError(layout)


def build(
    cfg: Config,
    device: torch.device | str = "cuda",
    *,
    head_lo: int = 0,
    head_hi: int | None = None,
    layout: str = "nhd",
    seed: int = 0,
    extra_blocks: int = 16,
) -> Workload:
    """Allocate and fill one rank's store and paged cache for ``cfg`` on ``device``."""
    device = torch.device(device)
    head_hi = cfg.heads if head_hi is None else head_hi
    h = head_hi - head_lo
    d, bs = cfg.head_size, cfg.block_size
    scales = _channel_scales(cfg, seed)[:, head_lo:head_hi].to(device)
    gen = torch.Generator(device=device).manual_seed(seed + 1000 * head_lo + 17)
    fp8 = cfg.dtype == "e4m3"
    k_scales = v_scales = None
    if fp8:
        g = torch.Generator().manual_seed(seed + 3)
        k_scales = (0.01 + 0.09 * torch.rand(cfg.layers, generator=g)).to(device)
        v_scales = (0.01 + 0.09 * torch.rand(cfg.layers, generator=g)).to(device)
    store_dtype = torch.float8_e4m3fn if fp8 else torch.bfloat16

    stores: list[list[torch.Tensor]] = []
    for cap in cfg.history:
        per_layer = []
        for li in range(cfg.layers):
            x = torch.randn(cap, h, 2 * d, device=device, generator=gen) * scales[li]
            if fp8:
                q = torch.empty_like(x)
                q[..., :d] = x[..., :d] / k_scales[li]
                q[..., d:] = x[..., d:] / v_scales[li]
                per_layer.append(q.clamp_(-448.0, 448.0).to(store_dtype))
            else:
                per_layer.append(x.to(store_dtype))
            del x
        stores.append(per_layer)

    # destination blocks: each session gets its own seeded permutation of free blocks
    rng = np.random.default_rng(seed + 99)
    need = []
    for si, segs in enumerate(cfg.segments):
        end = max(s.dst_end for s in segs)
        blocks = -(-end // bs)
        free = cfg.free_blocks[si] if si < len(cfg.free_blocks) else blocks + extra_blocks
        need.append((blocks, max(free, blocks)))
    total_blocks = sum(f for _, f in need)
    order = rng.permutation(total_blocks)
    tables_host, at = [], 0
    for blocks, free in need:
        tables_host.append(order[at : at + free][:blocks].astype(np.int32))
        at += free
    kv = [
        torch.zeros(_paged_shape(layout, total_blocks, bs, h, d), dtype=store_dtype, device=device)
        for _ in range(cfg.layers)
    ]
    tables = [torch.from_numpy(t).to(device) for t in tables_host]
    runs = []
    for si, segs in enumerate(cfg.segments):
        for s in segs:
            runs.append(RunSpec(session=si, store_start=s.src_start, length=s.length,
                                delta=s.delta, block_table=tables[si], paged_start=s.dst_start))
    inv = inv_freq(cfg.head_size, cfg.theta).to(device)
    return Workload(cfg, head_lo, head_hi, stores, kv, layout, tables, tables_host, runs, inv,
                    k_scales, v_scales)
