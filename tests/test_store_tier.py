"""The store tier off the GPU (pinned host memory, or another GPU): staged copies.

CPU tests cover the chunk planner and the store bookkeeping on a host device.
GPU tests load and save through :class:`ShiftWorker` with the store in pinned
host memory and compare the paged caches / store rows bit for bit with the
same jobs against a device store (itself checked against the oracle in
``test_gpu_parity.py``), and with the oracle directly for one case.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from marathon_b200 import shift_kernels as sk
from marathon_b200.shift_kernels import ShiftError
from marathon_b200.shift_store import ShiftStore
from marathon_b200.store_tier import is_staged, plan_chunks
from marathon_b200.worker import LoadJob, SaveJob, ShiftWorker
from oracle import shift_oracle as O
from parity import reference_tables

H, D, BS = 8, 128, 16
ROW = H * 2 * D * 2  # bytes of one bf16 store row


# --------------------------------------------------------------- planner (CPU)
def _covered(chunks, lengths, n_layers):
    seen = {}
    for ch in chunks:
        for li in range(ch.first_layer, ch.first_layer + ch.n_layers):
            for p in ch.pieces:
                for t in range(p.offset, p.offset + p.length):
                    key = (li, p.run, t)
                    assert key not in seen, f"{key} staged twice"
                    seen[key] = True
    assert len(seen) == n_layers * sum(lengths)


@pytest.mark.parametrize("chunk_rows", [1, 3, 64, 445, 446, 447, 900, 1338, 10_000])
def test_plan_chunks_covers_every_row_once_within_the_budget(chunk_rows):
    lengths, n_layers = [190, 9, 97, 150], 3
    chunks = plan_chunks(lengths, ROW, n_layers, chunk_rows * ROW)
    _covered(chunks, lengths, n_layers)
    for ch in chunks:
        assert ch.nbytes <= max(chunk_rows, 1) * ROW
        sizes = [p.length * ROW for p in ch.pieces]
        assert ch.offsets == list(np.cumsum([0] + sizes[:-1]))  # dense, row aligned
        assert ch.layer_bytes == sum(sizes)
        assert all(o % 16 == 0 for o in ch.offsets)
    if chunk_rows >= sum(lengths):  # whole layers per chunk; the first holds one
        per = chunk_rows // sum(lengths)
        assert chunks[0].n_layers == 1
        assert len(chunks) == (1 + -(-(n_layers - 1) // per) if per > 1 else n_layers)
        assert all(len(ch.pieces) == len(lengths) for ch in chunks)
    else:
        assert all(ch.n_layers == 1 for ch in chunks)


def test_plan_chunks_random_lengths():
    rng = np.random.default_rng(3)
    for _ in range(50):
        lengths = rng.integers(1, 300, size=rng.integers(1, 9)).tolist()
        n_layers = int(rng.integers(1, 6))
        chunk = int(rng.integers(1, 2000)) * ROW + int(rng.integers(0, ROW))
        _covered(plan_chunks(lengths, ROW, n_layers, chunk), lengths, n_layers)


def test_plan_chunks_rejects_bad_input():
    with pytest.raises(ShiftError):
        plan_chunks([10], 24, 2)  # rows not a multiple of 16 bytes
    with pytest.raises(ShiftError):
        plan_chunks([10, 0], ROW, 2)
    with pytest.raises(ShiftError):
        plan_chunks([], ROW, 2)
    with pytest.raises(ShiftError):
        plan_chunks([4], ROW, 0)


def test_which_stores_are_staged():
    dev = torch.device("cuda", 0)
    assert is_staged("cpu", dev)
    assert not is_staged("cuda", dev)
    assert not is_staged("cuda:0", dev)
    assert is_staged("cuda:1", dev)
    with pytest.raises(ShiftError):
        is_staged("meta", dev)


def test_host_store_bookkeeping_matches_device_semantics():
    """The same reserve/write/read rules on a host-resident store (no GPU needed)."""
    st = ShiftStore(budget_tokens=4096, device="cpu", slab=64)
    assert st.reserve("s", 16, 100)
    rows = torch.arange(100 * 4, dtype=torch.float32).reshape(100, 1, 4)
    st.write("s", "l0", 16, rows)
    got = st.read("s", "l0", 20, 10)
    assert got.device.type == "cpu" and torch.equal(got, rows[4:14])
    assert st.reserve("s", 116, 200)  # growth keeps [0, filled)
    assert torch.equal(st.read("s", "l0", 16, 100), rows)
    assert st.capacity("s") >= 316


# ---------------------------------------------------------------- GPU paths
def _rand(shape, fp8, g):
    x = torch.randn(shape, generator=g)
    if fp8:
        return (x * 20).clamp(-448, 448).to(torch.float8_e4m3fn)
    return x.to(torch.bfloat16)


def _case(cuda, store_device, *, fp8=False, layers=3, chunk_bytes=None, seed=0):
    """Three sessions in a store on ``store_device``; caches and jobs on ``cuda``."""
    g = torch.Generator().manual_seed(seed)
    nblk = 48
    names = [f"layer.{i}" for i in range(layers)]
    caps = [400, 260, 500]
    host_rows = [[_rand((c, H, 2 * D), fp8, g) for _ in range(layers)] for c in caps]
    kv_host = [_rand((nblk, BS, H, 2 * D), fp8, g) for _ in range(layers)]
    store = ShiftStore(budget_tokens=sum(caps), device=store_device)
    for si, rows in enumerate(host_rows):
        bufs = {}
        for n, t in zip(names, rows, strict=True):
            b = store.new_buffer(t.shape, t.dtype, store_device)
            b.copy_(t)
            bufs[n] = b
        store.adopt(f"s{si}", bufs, 0, caps[si])
    kv = [t.to(cuda) for t in kv_host]
    k_scales = torch.tensor([0.031, 0.07, 0.012, 0.05][:layers], dtype=torch.float32)
    kw = {} if chunk_bytes is None else {"chunk_bytes": chunk_bytes}
    worker = ShiftWorker(store, BS, sk.inv_freq(D, 1e6), layout="nhd", fp8=fp8,
                         k_scales=k_scales if fp8 else None, **kw)
    worker.register(dict(zip(names, kv, strict=True)))
    perm = np.random.default_rng(seed).permutation(nblk).astype(np.int32)
    slots = torch.from_numpy(O.slots(perm[26:40], 7, 7 + 97, BS)).to(cuda)
    jobs = [
        LoadJob("s0", 3, 37, 19, 190, block_ids=perm[:14]),
        LoadJob("s1", 250, -250, 0, 9, block_ids=perm[14:26]),
        LoadJob("s2", 401, 6759, 7, 97, slots=slots),
        LoadJob("s1", 10, 0, 30, 150, block_ids=perm[14:26]),
    ]
    return worker, kv, host_rows, jobs, k_scales


def _bits(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.uint8).numpy() if t.dtype == torch.float8_e4m3fn else \
        t.view(torch.int16).numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_rows", [None, 446, 80, 10])
@pytest.mark.parametrize("fp8", [False, True])
def test_host_tier_load_matches_device_store(cuda, fp8, chunk_rows):
    chunk = None if chunk_rows is None else chunk_rows * H * 2 * D * (1 if fp8 else 2)
    host_w, host_kv, _, jobs, _ = _case(cuda, "cpu", fp8=fp8, chunk_bytes=chunk, seed=11)
    dev_w, dev_kv, _, djobs, _ = _case(cuda, str(cuda), fp8=fp8, seed=11)
    assert host_w.mover is not None and dev_w.mover is None
    assert len(host_w.load(jobs)) == len(jobs)
    assert len(dev_w.load(djobs)) == len(djobs)
    torch.cuda.synchronize()
    if chunk_rows is not None:
        assert host_w.mover.last_chunks > 1
    for a, b in zip(host_kv, dev_kv, strict=True):
        assert np.array_equal(_bits(a), _bits(b))
    # counters and LRU order follow the same rules as the device store
    assert host_w.store.loaded_token_layers == dev_w.store.loaded_token_layers


@pytest.mark.gpu
def test_host_tier_load_vs_oracle(cuda):
    worker, kv, host_rows, jobs, _ = _case(cuda, "cpu", chunk_bytes=100 * ROW, seed=4)
    before = [_bits(t).reshape(-1).copy() for t in kv]
    worker.load(jobs)
    torch.cuda.synchronize()
    deltas = sorted({j.delta for j in jobs if j.delta})
    tables = reference_tables(deltas, sk.inv_freq(D, 1e6).numpy(), cuda)
    runs = []
    for j in jobs:
        r = {"session": int(j.session[1:]), "store_start": j.src_start, "len": j.length,
             "table": deltas.index(j.delta) if j.delta else -1}
        if j.slots is not None:
            r["slots"] = j.slots.cpu().numpy()
        else:
            r["block_table"], r["paged_start"] = np.asarray(j.block_ids), j.dst_start
        runs.append(r)
    st = [[_bits(t) for t in per] for per in host_rows]
    blk, off, head = BS * H * 2 * D, H * 2 * D, 2 * D
    paged = [O.Paged(b, 0, D, blk, off, head, BS, H, D) for b in before]
    O.load(st, runs, paged, tables, O.BF16, None)
    for li, t in enumerate(kv):
        assert np.array_equal(_bits(t).reshape(-1), paged[li].flat), li


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_rows", [None, 120])
def test_host_tier_save_matches_device_store(cuda, chunk_rows):
    chunk = None if chunk_rows is None else chunk_rows * ROW
    host_w, _, _, jobs, _ = _case(cuda, "cpu", chunk_bytes=chunk, seed=21)
    dev_w, _, _, djobs, _ = _case(cuda, str(cuda), seed=21)
    names = host_w.layers.names
    saves = [SaveJob(j.session, j.dst_start, j.length, block_ids=j.block_ids, slots=j.slots)
             for j in jobs]
    dsaves = [SaveJob(j.session, j.dst_start, j.length, block_ids=j.block_ids, slots=j.slots)
              for j in djobs]
    assert host_w.save(saves) == dev_w.save(dsaves)
    # a middle layer alone (the per-layer save shape)
    host_w.save(saves[:2], names[1:2])
    dev_w.save(dsaves[:2], names[1:2])
    torch.cuda.synchronize()
    for s in ("s0", "s1", "s2"):
        for n in names:
            a = host_w.store._sessions[s].layers[n]
            b = dev_w.store._sessions[s].layers[n]
            assert a.device.type == "cpu" and a.is_pinned()
            assert np.array_equal(_bits(a), _bits(b)), (s, n)


@pytest.mark.gpu
def test_host_tier_bad_slot_raises_after_the_batch(cuda):
    worker, kv, _, jobs, _ = _case(cuda, "cpu", chunk_bytes=64 * ROW, seed=2)
    bad = jobs[2].slots.clone()
    bad[5] = 48 * BS + 3  # past the paged cache
    jobs[2].slots = bad
    with pytest.raises(ShiftError, match="slot outside"):
        worker.load(jobs)
    torch.cuda.synchronize()  # the context is still usable
    assert torch.isfinite(kv[0].float()).all()


@pytest.mark.gpu
def test_host_tier_store_range_checked_on_host(cuda):
    worker, _, _, jobs, _ = _case(cuda, "cpu", seed=3)
    view = worker.store.view(["s1"], worker.layers.names)
    run = sk.RunSpec(0, 250, 20, 5, block_table=np.arange(4, dtype=np.int32), paged_start=0)
    with pytest.raises(ShiftError, match="outside capacity"):
        worker.mover.load([run], view, worker.inv)


@pytest.mark.gpu
def test_peer_gpu_store_tier(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    host_w, host_kv, _, jobs, _ = _case(cuda, "cuda:1", chunk_bytes=150 * ROW, seed=8)
    dev_w, dev_kv, _, djobs, _ = _case(cuda, str(cuda), seed=8)
    assert host_w.mover is not None
    host_w.load(jobs)
    dev_w.load(djobs)
    torch.cuda.synchronize()
    for a, b in zip(host_kv, dev_kv, strict=True):
        assert np.array_equal(_bits(a), _bits(b))


@pytest.mark.gpu
def test_host_tier_async_load_layer_by_layer(cuda):
    """An asynchronous staged load, consumed layer by layer on the current stream
    (as a forward pass would), lands the same bits as the device store."""
    host_w, host_kv, _, jobs, _ = _case(cuda, "cpu", layers=4, chunk_bytes=200 * ROW, seed=13)
    dev_w, dev_kv, _, djobs, _ = _case(cuda, str(cuda), layers=4, seed=13)
    dev_w.load(djobs)
    assert len(host_w.load(jobs, asynchronous=True)) == len(jobs)
    assert host_w.pending is not None and host_w.mover.last_chunks > 4
    snaps = []
    for name, t in zip(host_w.layers.names, host_kv, strict=True):
        host_w.wait_layer(name)
        snaps.append(t.clone())  # ordered after exactly this layer's rows
    host_w.finish_pending()
    assert host_w.pending is None
    torch.cuda.synchronize()
    for a, b in zip(snaps, dev_kv, strict=True):
        assert np.array_equal(_bits(a), _bits(b))


@pytest.mark.gpu
def test_host_tier_async_load_reports_bad_slots_at_finish(cuda):
    worker, _, _, jobs, _ = _case(cuda, "cpu", chunk_bytes=64 * ROW, seed=5)
    bad = jobs[2].slots.clone()
    bad[0] = -1
    jobs[2].slots = bad
    worker.load(jobs, asynchronous=True)
    with pytest.raises(ShiftError, match="slot outside"):
        worker.finish_pending()
    assert worker.pending is None


@pytest.mark.gpu
def test_device_store_queued_load_checks_status_at_finish(cuda):
    """A device store's asynchronous load: same bits as the blocking load, and a
    rejected token surfaces at ``finish_pending``."""
    a_w, a_kv, _, jobs, _ = _case(cuda, str(cuda), seed=17)
    b_w, b_kv, _, bjobs, _ = _case(cuda, str(cuda), seed=17)
    a_w.load(jobs, asynchronous=True)
    assert a_w.pending is not None
    b_w.load(bjobs)
    a_w.finish_pending()
    torch.cuda.synchronize()
    for x, y in zip(a_kv, b_kv, strict=True):
        assert np.array_equal(_bits(x), _bits(y))
    bad = jobs[2].slots.clone()
    bad[3] = 48 * BS + 1
    jobs[2].slots = bad
    a_w.load(jobs, asynchronous=True)
    with pytest.raises(ShiftError, match="slot outside"):
        a_w.finish_pending()


def test_chunk_copies_and_slot_view_agree():
    """The copy records of a chunk move exactly each piece's store rows of each
    layer, and the slot view the kernel reads points at where they land."""
    from marathon_b200.shift_kernels import RunSpec, StoreView
    from marathon_b200.store_tier import StagedMover

    rng = np.random.default_rng(2)
    lengths = [190, 9, 97, 150]
    runs = [RunSpec(i % 2, int(rng.integers(0, 100)), n, 5, block_table=np.arange(30),
                    paged_start=0) for i, n in enumerate(lengths)]
    n_layers = 3
    ptrs = (np.arange(2 * n_layers, dtype=np.uint64).reshape(2, n_layers) + 1) * (1 << 30)
    view = StoreView(ptrs, np.array([400, 400], np.int64), 8 * 256, 256)
    base = 1 << 44
    for chunk_rows in (10_000, 300, 64):
        for ch in plan_chunks(lengths, ROW, n_layers, chunk_rows * ROW):
            rec = StagedMover._copies(ch, runs, view, ROW, base, to_slot=True)
            sv = StagedMover._slot_view(ch, base, view)
            assert sv.ptrs.shape == (len(ch.pieces), ch.n_layers)
            i = 0
            for li in range(ch.n_layers):
                for j, p in enumerate(ch.pieces):
                    r = runs[p.run]
                    want_src = int(view.ptrs[r.session, ch.first_layer + li]) + \
                        (r.store_start + p.offset) * ROW
                    assert int(rec["src"][i]) == want_src
                    assert int(rec["dst"][i]) == int(sv.ptrs[j, li])  # kernel reads row 0
                    assert int(rec["bytes"][i]) == p.length * ROW
                    assert sv.caps[j] == p.length
                    i += 1
            assert i == len(rec)
            # a save copies the other way over the same ranges
            back = StagedMover._copies(ch, runs, view, ROW, base, to_slot=False)
            assert np.array_equal(back["src"], rec["dst"]) and np.array_equal(back["dst"], rec["src"])
