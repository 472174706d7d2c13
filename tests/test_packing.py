"""Descriptor packing on the host, without a GPU.

The launcher packs a batch into one staging buffer by two routes -- record by
record for a few runs, column-wise with numpy for many -- and the kernels
read the result as ``mshift_run`` records, a store pointer table, capacities,
deltas and block tables.  Both routes must write the same bytes, and the
records must say what the runs said (tile prefixes as ``mshift_plan_tiles``
computes them, table indices by delta, block tables copied beside them).
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from marathon_b200 import _lib
from marathon_b200.shift_kernels import Launcher, RunSpec, StoreView

BASE = 0x7F0000000000  # the fake device address of the staging slot


class _FakeStaging:
    def __init__(self) -> None:
        self.host = np.zeros(1 << 20, dtype=np.uint8)
        self.total = 0

    def begin(self, n: int):
        self.host[:] = 0xAB  # stale bytes: packing must overwrite every byte it claims
        return 0, self.host, BASE

    def upload(self, slot: int, n: int, stream_ptr: int) -> None:
        self.total = n

    def finish(self, slot: int, stream) -> None:
        self.finished = slot


class _FakeSlots:
    """Stands in for a CUDA int64 slot tensor (only its address is packed)."""

    dtype = torch.int64
    is_cuda = True

    def __init__(self, n: int, addr: int) -> None:
        self.n, self.addr = n, addr

    def numel(self) -> int:
        return self.n

    def data_ptr(self) -> int:
        return self.addr


def _launcher(heads: int, small: int, dtype: int = _lib.BF16) -> Launcher:
    la = object.__new__(Launcher)
    la.geo = SimpleNamespace(heads=heads, dtype=dtype)
    la.lib = _lib.load()
    la.fixed_tile = False
    la.tile_tokens = int(la.lib.mshift_default_tile_tokens(heads))
    la._grid = 296
    la.staging = _FakeStaging()
    la.last_h2d = 0
    la._SMALL = small
    la.EARLY_UPLOAD = False  # no copy stream without a GPU
    return la


def _batch(seed: int):
    rng = np.random.default_rng(seed)
    n_sessions, n_layers = int(rng.integers(1, 5)), int(rng.integers(1, 6))
    tables = [rng.permutation(200)[: int(rng.integers(20, 60))].astype(np.int32)
              for _ in range(n_sessions)]
    runs = []
    for i in range(int(rng.integers(1, 40))):
        s = int(rng.integers(0, n_sessions))
        n = int(rng.integers(1, 300))
        delta = int(rng.choice([0, 7, -40, 186]))
        if rng.random() < 0.25:
            runs.append(RunSpec(s, int(rng.integers(0, 500)), n, delta,
                                slots=_FakeSlots(n, 0x6000_0000 + 4096 * i)))
        else:
            runs.append(RunSpec(s, int(rng.integers(0, 500)), n, delta, block_table=tables[s],
                                paged_start=int(rng.integers(0, 100))))
    ptrs = rng.integers(1, 2**40, size=(n_sessions, n_layers)).astype(np.uint64) * 16
    caps = rng.integers(500, 2000, size=n_sessions).astype(np.int64)
    view = StoreView(ptrs, caps, 8 * 256, 256)
    deltas = sorted({r.delta for r in runs if r.delta})
    return runs, view, deltas, n_layers


@pytest.mark.parametrize("seed", range(12))
def test_record_and_column_packing_write_the_same_bytes(seed):
    runs, view, deltas, n_layers = _batch(seed)
    stream = SimpleNamespace(cuda_stream=0)
    a, b = _launcher(8, small=10**9), _launcher(8, small=0)
    pa = a._prepare("load", runs, view, deltas, 0, n_layers, stream)
    pb = b._prepare("load", runs, view, deltas, 0, n_layers, stream)
    assert pa.h2d_bytes == pb.h2d_bytes == a.staging.total == b.staging.total
    assert (pa.tiles, pa.tile_tokens, pa.n_runs) == (pb.tiles, pb.tile_tokens, pb.n_runs)
    assert (pa.runs, pa.ptrs, pa.caps, pa.deltas) == (pb.runs, pb.ptrs, pb.caps, pb.deltas)
    assert a.staging.host[: pa.h2d_bytes].tobytes() == b.staging.host[: pb.h2d_bytes].tobytes()


@pytest.mark.parametrize("seed", range(6))
def test_packed_records_describe_the_runs(seed):
    runs, view, deltas, n_layers = _batch(100 + seed)
    la = _launcher(8, small=10**9)
    p = la._prepare("load", runs, view, deltas, 0, n_layers, SimpleNamespace(cuda_stream=0))
    host = la.staging.host
    assert host[:16].tobytes() == bytes(16)  # the error word starts at zero
    off = p.runs - BASE
    rec = host[off : off + 56 * len(runs)].view(_lib.RUN_DTYPE)
    # tile prefixes exactly as the library's own planner computes them
    plan = np.zeros(len(runs), dtype=_lib.RUN_DTYPE)
    plan["len"] = [r.length for r in runs]
    tiles = la.lib.mshift_plan_tiles(plan.ctypes.data, len(runs), p.tile_tokens)
    assert tiles == p.tiles and np.array_equal(plan["tile_begin"], rec["tile_begin"])
    for r, x in zip(runs, rec, strict=True):
        assert (x["store_start"], x["len"], x["session"]) == (r.store_start, r.length, r.session)
        assert x["table"] == (deltas.index(r.delta) if r.delta else -1)
        if r.slots is not None:
            assert x["slots"] == r.slots.data_ptr() and x["block_table"] == 0
            continue
        assert x["slots"] == 0 and x["paged_start"] == r.paged_start
        t_off = int(x["block_table"]) - BASE
        assert t_off % 16 == 0 and x["block_table_len"] == r.block_table.size
        got = host[t_off : t_off + 4 * r.block_table.size].view(np.int32)
        assert np.array_equal(got, r.block_table)
    ptrs = host[p.ptrs - BASE : p.ptrs - BASE + view.ptrs.nbytes].view(np.uint64)
    assert np.array_equal(ptrs.reshape(view.ptrs.shape), view.ptrs)
    caps = host[p.caps - BASE : p.caps - BASE + view.caps.nbytes].view(np.int64)
    assert np.array_equal(caps, view.caps)
    if deltas:
        d = host[p.deltas - BASE : p.deltas - BASE + 8 * len(deltas)].view(np.int64)
        assert d.tolist() == deltas


@pytest.mark.parametrize("heads,tokens,layers,want", [
    (8, 28_608, 40, 56),    # full c2 turn: 121 tiles of 256 units per CTA -> 448 units
    (4, 28_608, 40, 64),    # a TP2 rank's share: 60 per CTA -> 256 units
    (2, 28_608, 40, 128),
    (1, 28_608, 40, 256),   # a TP8 rank's share
    (1, 600_000, 40, 448),  # one head, but a long batch
    (64, 1_000, 4, 16),     # many heads: the 16-token floor
    (8, 10, 1, 32),         # a tiny batch
])
def test_tile_rule(heads, tokens, layers, want):
    la = _launcher(heads, small=32)
    assert la._tile_for(tokens, layers) == want


@pytest.mark.parametrize("heads,want", [(8, 48), (4, 96), (2, 192), (1, 384)])
def test_tile_rule_e4m3_is_whole_tma_stages(heads, want):
    """384 units of 256 bytes: four 24 KiB stages of the TMA kernel at any head count."""
    la = _launcher(heads, small=32, dtype=_lib.E4M3)
    assert la._tile_for(28_608, 40) == want
    assert want * heads * 256 == 4 * 24 * 1024
