"""Head-sharded shift on 2 ranks over gloo (CPU): no exchange needed, one table broadcast.

Each rank computes the oracle shift of its own KV-head shard; gathering the
shards (for verification only) reproduces the unsharded result bit for bit,
which is the property that lets the GPU path run with no data collective.
A rank that never joins the broadcast ends the other rank's call with an
error within the process group's timeout rather than a hang.
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from marathon_b200.sharding import (
    broadcast_table,
    head_shard,
    pack_table,
    shard_rows,
    unpack_table,
)
from oracle import shift_oracle as O

H, D, BS = 8, 32, 4


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    rng = np.random.default_rng(12)
    store = rng.integers(0, 2**16, (50, H, 2 * D), dtype=np.uint16)
    store &= np.uint16(0xBFFF)  # keep exponents finite (no inf/nan bf16 patterns)
    runs = [
        {"session": 0, "store_start": 2, "length": 30, "delta": 7, "paged_start": 9},
        {"session": 0, "store_start": 40, "length": 9, "delta": -40, "paged_start": 0},
    ]
    table = np.random.default_rng(3).permutation(16).astype(np.int64)
    return store, runs, table


def _shift(store, runs, table, heads_lo, heads_hi):
    h = heads_hi - heads_lo
    nblk = 16
    flat = np.zeros(nblk * BS * h * 2 * D, dtype=np.uint16)
    paged = O.Paged(flat, 0, D, BS * h * 2 * D, h * 2 * D, 2 * D, BS, h, D)
    inv = O.inv_freq(D, 1e6)
    part = shard_rows(store, heads_lo, heads_hi)
    for r in runs:
        rows = part[r["store_start"] : r["store_start"] + r["length"]]
        sl = O.slots(table, r["paged_start"], r["paged_start"] + r["length"], BS)
        O.scatter_shifted(rows, paged, sl, O.rope_tables([r["delta"]], inv)[0], O.BF16)
    return flat.reshape(nblk, BS, h, 2 * D)


def _worker(rank, world, port, mode, out):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=5))
        store, runs, table = _case()
        if mode == "absent" and rank == 1:
            return  # never joins the broadcast
        objs = [type("R", (), r) for r in runs]
        mine = pack_table(objs) if rank == 0 else None
        try:
            got = broadcast_table(mine, len(runs))
        except Exception as e:  # noqa: BLE001 - the failure is what this mode tests
            out.put((rank, "error", repr(e)))
            return
        assert unpack_table(got) == runs
        lo, hi = head_shard(H, rank, world)
        shard = torch.from_numpy(_shift(store, unpack_table(got), table, lo, hi).astype(np.int32))
        parts = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(parts, shard)  # verification only: not part of the shift path
        out.put((rank, "ok", torch.cat(parts, dim=2).numpy()))
    except Exception:  # noqa: BLE001
        out.put((rank, "crash", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2 if mode == "ok" else 1):
        rank, status, payload = out.get(timeout=120)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_head_shards_partition_the_heads():
    for world in (1, 2, 4, 8):
        spans = [head_shard(8, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 8
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:], strict=False))
    with pytest.raises(ValueError):
        head_shard(8, 0, 3)


def test_two_ranks_shift_their_own_heads_and_agree_with_the_whole():
    results = _run("ok")
    store, runs, table = _case()
    whole = _shift(store, runs, table, 0, H).astype(np.int32)
    for rank in (0, 1):
        status, payload = results[rank]
        assert status == "ok", payload
        assert np.array_equal(payload, whole)


def test_a_rank_that_never_arrives_is_an_error_not_a_hang():
    results = _run("absent")
    status, payload = results[0]
    assert status == "error", payload
