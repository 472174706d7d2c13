"""The allocation-free batched load, checked against the allocating entry points.

``mshift_load_noalloc`` serves callers that cannot allocate device memory
while they serve: a server whose device pool is divided up once at start-up
(every byte already belongs to the KV cache and the store), or a host binding
that can only hand over pointers it already owns.  It keeps the batch's
rotation tables in a fixed array inside the library instead of a buffer the
caller would have to provide.  This test drives it through the C ABI on two
consecutive calls with different delta sets — so a stale table left by the
first call would show up in the second — and requires the paged caches it
writes to be bit-identical to what ``mshift_rope_tables`` + ``mshift_load``
write from the same inputs (the exactness the other parity tests hold the
kernels to).  It also checks the documented limit is enforced before any
launch.  The file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from marathon_b200 import _lib
from marathon_b200.shift_kernels import inv_freq

pytestmark = pytest.mark.gpu

H, D, BS, L, NBLK = 8, 128, 16, 3, 64


def _runs(tables_of_runs, bt_ptr, bt_len):
    """Four runs over two sessions; ``tables_of_runs`` gives each run's delta index."""
    spec = [  # session, store_start, len, paged_start
        (0, 5, 200, 40),
        (1, 0, 33, 300),
        (0, 230, 64, 500),
        (1, 100, 150, 640),
    ]
    rec = np.zeros(len(spec), dtype=_lib.RUN_DTYPE)
    for i, ((s, a, n, p), t) in enumerate(zip(spec, tables_of_runs, strict=True)):
        rec[i]["session"], rec[i]["store_start"], rec[i]["len"] = s, a, n
        rec[i]["paged_start"], rec[i]["table"] = p, t
        rec[i]["block_table"], rec[i]["block_table_len"] = bt_ptr, bt_len
    lib = _lib.load()
    tiles = lib.mshift_plan_tiles(rec.ctypes.data, len(rec), 32)
    assert tiles > 0
    return rec, tiles


@pytest.mark.parametrize("rotary", [128, 64], ids=["full-rotary", "partial-rotary"])
def test_noalloc_load_matches_the_allocating_entry_points(cuda, rotary):
    lib = _lib.load()
    g = torch.Generator().manual_seed(21)
    stores = [[torch.randn(400, H, 2 * D, generator=g).to(torch.bfloat16).to(cuda)
               for _ in range(L)] for _ in range(2)]
    base = [torch.randn(NBLK, BS, H, 2 * D, generator=g).to(torch.bfloat16) for _ in range(L)]
    kv_ref = [t.to(cuda) for t in base]
    kv_new = [t.to(cuda) for t in base]
    bt = torch.from_numpy(np.random.default_rng(4).permutation(NBLK).astype(np.int32)).to(cuda)

    store_ptrs = torch.tensor([t.data_ptr() for per in stores for t in per], dtype=torch.int64,
                              device=cuda)
    caps = torch.tensor([400, 400], dtype=torch.int64, device=cuda)
    k_ref = torch.tensor([t.data_ptr() for t in kv_ref], dtype=torch.int64, device=cuda)
    v_ref = k_ref + D * 2
    k_new = torch.tensor([t.data_ptr() for t in kv_new], dtype=torch.int64, device=cuda)
    v_new = k_new + D * 2
    inv = inv_freq(rotary, 1e6).to(cuda)
    half = rotary // 2
    err = torch.zeros(2, dtype=torch.int32, device=cuda)
    paged = _lib.Paged(BS * H * 2 * D, H * 2 * D, 2 * D, NBLK, BS, H, D, _lib.BF16)
    stream = torch.cuda.current_stream(cuda).cuda_stream

    # two calls in a row: different numbers of deltas, different values
    calls = [([186, -566, 37], [0, 1, 2, 0]), ([10000, -4], [1, -1, 0, 1])]
    for deltas, which in calls:
        d = torch.tensor(deltas, dtype=torch.int64, device=cuda)
        rec, tiles = _runs(which, bt.data_ptr(), bt.numel())
        runs = torch.from_numpy(rec.view(np.uint8).copy()).to(cuda)

        tables = torch.empty(len(deltas), 2, half, dtype=torch.float32, device=cuda)
        _lib.check(lib.mshift_rope_tables(d.data_ptr(), len(deltas), inv.data_ptr(), half,
                                          tables.data_ptr(), stream), "tables")
        _lib.check(lib.mshift_load(paged, rotary, runs.data_ptr(), len(rec), 32, tiles, L,
                                   store_ptrs.data_ptr(), caps.data_ptr(), 2, H * 2 * D, 2 * D,
                                   k_ref.data_ptr(), v_ref.data_ptr(), tables.data_ptr(),
                                   len(deltas), None, err.data_ptr(), stream), "load")
        _lib.check(lib.mshift_load_noalloc(paged, rotary, runs.data_ptr(), len(rec), 32, tiles, L,
                                           store_ptrs.data_ptr(), caps.data_ptr(), 2, H * 2 * D,
                                           2 * D, k_new.data_ptr(), v_new.data_ptr(),
                                           d.data_ptr(), len(deltas), inv.data_ptr(), None,
                                           err.data_ptr() + 4, stream), "load_noalloc")
        torch.cuda.synchronize()
        assert err.tolist() == [0, 0]
        for a, b in zip(kv_ref, kv_new, strict=True):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        # and the call really moved something
        assert not torch.equal(kv_new[0].cpu().view(torch.int16), base[0].view(torch.int16))


def test_noalloc_rejects_more_deltas_than_its_scratch_holds(cuda):
    lib = _lib.load()
    limit = lib.mshift_noalloc_max_deltas()
    assert limit == 256
    kv = torch.zeros(NBLK, BS, H, 2 * D, dtype=torch.bfloat16, device=cuda)
    before = kv.clone()
    paged = _lib.Paged(BS * H * 2 * D, H * 2 * D, 2 * D, NBLK, BS, H, D, _lib.BF16)
    d = torch.zeros(limit + 1, dtype=torch.int64, device=cuda)
    p = ctypes.c_void_p(kv.data_ptr())
    rc = lib.mshift_load_noalloc(paged, D, p, 1, 32, 1, 1, p, p, 1, H * 2 * D, 2 * D, p, p,
                                 d.data_ptr(), limit + 1, p, None, p,
                                 torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _lib.ETOOBIG
    assert b"static scratch" in lib.mshift_strerror(rc)
    torch.cuda.synchronize()
    assert torch.equal(kv, before)


def test_noalloc_rejects_a_rotary_wider_than_its_scratch_rows(cuda):
    """Scratch rows hold rotary/2 <= 128 frequencies: rotary 258 is refused
    with MSHIFT_ETOOBIG before anything is launched, and the cache is unchanged."""
    lib = _lib.load()
    kv = torch.zeros(NBLK, BS, H, 2 * D, dtype=torch.bfloat16, device=cuda)
    before = kv.clone()
    paged = _lib.Paged(BS * H * 2 * D, H * 2 * D, 2 * D, NBLK, BS, H, D, _lib.BF16)
    d = torch.zeros(1, dtype=torch.int64, device=cuda)
    p = ctypes.c_void_p(kv.data_ptr())
    rc = lib.mshift_load_noalloc(paged, 258, p, 1, 32, 1, 1, p, p, 1, H * 2 * D, 2 * D, p, p,
                                 d.data_ptr(), 1, p, None, p,
                                 torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _lib.ETOOBIG
    torch.cuda.synchronize()
    assert torch.equal(kv, before)
