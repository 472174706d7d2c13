"""The vLLM connector: scheduler-side decisions on CPU, worker-side data path on the GPU.

vLLM objects are faked with the handful of attributes the connector reads
(the same fields the reference connector uses: ``req_id``, ``block_ids``,
``num_computed_tokens``, ``num_scheduled_tokens``, ``finished_req_ids``).
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

vllm_base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")
KVConnectorRole = vllm_base.KVConnectorRole

from marathon_b200 import vllm_shift_connector as C  # noqa: E402
from parity import reference_tables  # noqa: E402
from vllm_fakes import BS, fake_config, forward_context, new_req, request, sched_output  # noqa: E402,E501


def scheduler(extra=None):
    return C.MarathonShiftConnector(fake_config(extra or {"store_tokens": 65536}),
                                    KVConnectorRole.SCHEDULER, None)


def test_inv_freq_and_theta_follow_the_model_config():
    conn = scheduler()
    want = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    assert torch.equal(conn._inv_freq, want)
    cfg = fake_config()
    del cfg.model_config.hf_text_config.rope_theta
    cfg.model_config.hf_text_config.rope_parameters = {"rope_theta": 5e5}
    c2 = C.MarathonShiftConnector(cfg, KVConnectorRole.SCHEDULER, None)
    assert torch.equal(c2._inv_freq, 1.0 / (5e5 ** (torch.arange(0, 128, 2,
                                                                   dtype=torch.float32) / 128)))


def test_first_turn_saves_then_edit_turn_loads_shifted():
    conn = scheduler()
    # turn 0: 1000-token prompt, nothing to load, everything saved
    r0 = request("r0", {"session": "s", "save": True}, 1000)
    conn.on_new_request(r0)
    assert conn.get_num_new_matched_tokens(r0, 0) == (0, False)
    blocks0 = list(range(100, 100 + 63))
    meta = conn.build_connector_meta(sched_output([new_req("r0", blocks0, 0)], scheduled={"r0": 1000}))
    assert not meta.loads and len(meta.saves) == 1
    sv = meta.saves[0]
    assert (sv.session, sv.dst_start, sv.length) == ("s", 0, 1000)
    assert sv.slots.tolist() == (np.asarray(blocks0)[np.arange(1000) // BS] * BS
                                 + np.arange(1000) % BS).tolist()
    conn.request_finished(r0, blocks0)

    # turn 1: an edit at 200 grows 40 tokens by 24, the suffix [240, 1000) moves to [264, 1024)
    load = {"dst_start": 264, "dst_end": 1024, "delta": 24}
    r1 = request("r1", {"session": "s", "load": load, "save": "full"}, 1100)
    conn.on_new_request(r1)
    # vLLM's own prefix cache hit stops at 256 (block aligned, before the edit end)
    n, async_ = conn.get_num_new_matched_tokens(r1, 264 - 264 % BS + BS)
    assert async_ is False
    lo, hi = 272, 1024
    assert n == hi - lo
    conn.update_state_after_alloc(r1, None, n)
    blocks1 = list(range(300, 300 + 69))
    meta = conn.build_connector_meta(sched_output([new_req("r1", blocks1, hi)],
                                                  scheduled={"r1": 1100 - hi}))
    assert len(meta.loads) == 1
    ld = meta.loads[0]
    assert (ld.session, ld.src_start, ld.delta, ld.dst_start, ld.length) == ("s", lo - 24, 24, lo,
                                                                            hi - lo)
    # "full" widens the save to [0, hi) once ...
    assert (meta.saves[0].dst_start, meta.saves[0].length) == (0, 1100)
    # ... and is downgraded for the next (decode) step
    cached = SimpleNamespace(req_ids=["r1"], new_block_ids=[None], num_computed_tokens=[1100])
    meta2 = conn.build_connector_meta(sched_output(cached=cached, scheduled={"r1": 1}))
    assert (meta2.saves[0].dst_start, meta2.saves[0].length) == (1100, 1)


def test_extent_mode_saves_only_fresh_tokens_and_loads_by_generation():
    """``store_mode="extents"``: the reused tail keeps its generation-0 rows, the
    turn saves only what it computed, and a later turn loads from both."""
    from marathon_b200.extent_store import AddressBook

    conn = scheduler({"store_tokens": 65536, "store_mode": "extents"})
    book = AddressBook()
    # turn 0 (generation 0): 1000 tokens computed and saved
    r0 = request("r0", {"session": "s", "save": True, "gen": 0}, 1000)
    conn.on_new_request(r0)
    blocks0 = list(range(100, 100 + 63))
    meta = conn.build_connector_meta(sched_output([new_req("r0", blocks0, 0)],
                                                  scheduled={"r0": 1000}))
    assert [(sv.gen, sv.dst_start, sv.length) for sv in meta.saves] == [(0, 0, 1000)]
    conn.request_finished(r0, blocks0)
    assert book.after_turn([], 1000, 0) == []

    # turn 1 (generation 1): [200, 240) replaced by 64 tokens, tail [240, 1000) -> +24
    segs = [{"dst_start": 0, "dst_end": 200, "delta": 0},
            {"dst_start": 264, "dst_end": 1024, "delta": 24}]
    loads = book.loads(segs)
    dead = book.after_turn(segs, 1100, 1)
    r1 = request("r1", {"session": "s", "load": loads[1], "save": True, "gen": 1,
                        "release": [list(d) for d in dead]}, 1100)
    conn.on_new_request(r1)
    n, _ = conn.get_num_new_matched_tokens(r1, 192)  # vLLM's own prefix hit
    assert n == 0  # the load starts at 264, above the prefix hit: declined
    n, _ = conn.get_num_new_matched_tokens(r1, 272)
    assert n == 1024 - 272
    conn.update_state_after_alloc(r1, None, n)
    blocks1 = list(range(300, 300 + 69))
    meta = conn.build_connector_meta(sched_output([new_req("r1", blocks1, 1024)],
                                                  scheduled={"r1": 1100 - 1024}))
    assert meta.releases == [("s", 0, 200, 40)]
    ld = meta.loads[0]
    assert (ld.gen, ld.src_start, ld.delta, ld.dst_start, ld.length) == (0, 248, 24, 272, 752)
    # only the computed tail is saved, as generation 1 (no "full" rewrite)
    assert [(sv.gen, sv.dst_start, sv.length) for sv in meta.saves] == [(1, 1024, 76)]
    st = conn._store
    assert st.locate("s", 0, 200, 40, count=False) is None  # released
    assert st.locate("s", 0, 240, 760, count=False) is not None  # generation 0 intact
    conn.request_finished(r1, blocks1)


def test_load_is_declined_not_guessed_when_the_store_lost_the_source():
    conn = scheduler({"store_tokens": 4096})
    r = request("a", {"session": "x", "load": {"dst_start": 64, "dst_end": 640, "delta": 8}},
                700)
    conn.on_new_request(r)
    assert conn.get_num_new_matched_tokens(r, 64) == (0, False)  # nothing stored yet
    assert conn._store.misses == 1


def test_second_in_flight_writer_on_a_session_is_refused():
    conn = scheduler()
    conn.on_new_request(request("a", {"session": "s", "save": True}, 100))
    conn.on_new_request(request("b", {"session": "s", "save": True}, 100))
    assert conn._table.session_of("b") is None
    assert conn._table.conflicts == 1
    meta = conn.build_connector_meta(sched_output([new_req("b", [1, 2, 3, 4, 5, 6, 7], 0)],
                                                  scheduled={"b": 100}))
    assert meta.saves == []  # no session -> pass-through, no save


def test_stats_merges_instances():
    before = C.stats()["refusals"]
    conn = scheduler()
    conn._store.reserve("z", 0, 0)  # empty span: refused
    assert C.stats()["refusals"] == before + 1


# --------------------------------------------------------------- worker (GPU)
def _oracle_slots(blocks, lo, hi):
    from oracle import shift_oracle as O

    return O.slots(blocks, lo, hi, BS)


@pytest.mark.gpu
@pytest.mark.parametrize("shape_kind", ["split", "nhd", "hnd"])
@pytest.mark.parametrize("batch_save", [False, True])
@pytest.mark.parametrize("store_device", ["cuda", "cpu"])
def test_worker_save_then_shifted_load_through_the_connector(cuda, shape_kind, batch_save,
                                                              store_device):
    """Save a prompt layer by layer, then serve an edit turn's load: oracle-exact.

    With ``store_device="cpu"`` the store is pinned host memory: saves copy out
    through staging, and the load streams in asynchronously, each layer
    awaited through ``wait_for_layer_load`` as the forward pass would; with a
    device store the load is queued on the stream and checked at
    ``wait_for_save``.
    """
    from oracle import shift_oracle as O

    H, D, L, NBLK = 8, 128, 4, 96
    conn = C.MarathonShiftConnector(fake_config({"store_tokens": 8192,
                                                 "batch_save": batch_save,
                                                 "store_device": store_device,
                                                 "stage_chunk_bytes": 300 * H * 2 * D * 2}),
                                    KVConnectorRole.WORKER, None)
    g = torch.Generator().manual_seed(7)
    shapes = {"split": (2, NBLK, BS, H, D), "nhd": (NBLK, BS, H, 2 * D),
              "hnd": (NBLK, H, BS, 2 * D)}
    caches = {f"model.layers.{i}.self_attn.attn": torch.randn(shapes[shape_kind], generator=g)
              .to(torch.bfloat16).to(cuda) for i in range(L)}
    conn.register_kv_caches(caches)
    perm = np.random.default_rng(1).permutation(NBLK)
    blocks0 = perm[:40].tolist()

    # turn 0 saves [0, 600) from blocks0
    meta = C.ShiftConnectorMetadata(saves=[C._Save("s", 0, 600, blocks0, BS)])
    conn._store.reserve("s", 0, 600)  # the scheduler's reserve, mirrored
    conn.bind_connector_metadata(meta)
    for name, kv in caches.items():
        conn.save_kv_layer(name, kv, None)
    conn.wait_for_save()
    conn.clear_connector_metadata()
    torch.cuda.synchronize()
    entry = conn._store._sessions["s"]
    assert all(t.device.type == store_device for t in entry.layers.values())
    saved = {n: entry.layers[n][:600].clone() for n in caches}
    snap = {n: kv.clone() for n, kv in caches.items()}

    # turn 1: [64, 592) moves by +37 into a fresh block table
    blocks1 = perm[40:80].tolist()
    meta = C.ShiftConnectorMetadata(loads=[C._Load("s", 64, 37, 101, 528, blocks1, BS)])
    conn.bind_connector_metadata(meta)
    conn.start_load_kv(SimpleNamespace(no_compile_layers={}, virtual_engine=0))
    # the load is queued (status checked at the end of the step), as vLLM drives it
    assert conn._worker.pending is not None
    for name in caches:
        conn.wait_for_layer_load(name)
    conn.wait_for_save()
    assert conn._worker.pending is None
    conn.clear_connector_metadata()
    torch.cuda.synchronize()

    from marathon_b200.paged import describe

    inv = conn._inv_freq.numpy()
    tab = reference_tables([37], inv, cuda)[0]
    sl1 = _oracle_slots(blocks1, 101, 101 + 528)
    sl0 = _oracle_slots(blocks0, 0, 600)
    for name, kv in caches.items():
        geo = describe(kv, BS, conn._worker.layout)
        before = O.Paged(snap[name].cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1),
                         0, geo.v_offset, geo.blk_stride, geo.off_stride, geo.head_stride, BS, H, D)
        # the save must equal the paged rows it gathered
        k0, v0 = before.read(sl0)
        st = saved[name].cpu().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(st[..., :D], k0) and np.array_equal(st[..., D:], v0)
        # the load must equal the oracle's
        O.scatter_shifted(st[64:592], before, sl1, tab, O.BF16)
        got = kv.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1)
        assert np.array_equal(got, before.flat), name
    s = conn._store.stats()
    assert s["loaded_token_layers"] == 528 * L
    assert s["saved_token_layers"] == 600 * L


@pytest.mark.gpu
@pytest.mark.parametrize("store_device", ["cuda", "cpu"])
def test_extent_mode_three_turns_load_from_generation_zero(cuda, store_device):
    """Three turns through the worker hooks in ``store_mode="extents"``: the last
    turn loads spans first computed in turns 0 and 1, each rotated once from
    the bytes of the turn that computed it (bit-exact against the oracle)."""
    from oracle import shift_oracle as O

    H, D, L, NBLK = 8, 128, 3, 160
    conn = C.MarathonShiftConnector(fake_config({"store_tokens": 8192, "store_mode": "extents",
                                                 "store_device": store_device}),
                                    KVConnectorRole.WORKER, None)
    g = torch.Generator().manual_seed(3)
    caches = {f"model.layers.{i}.self_attn.attn":
              torch.randn(NBLK, BS, H, 2 * D, generator=g).to(torch.bfloat16).to(cuda)
              for i in range(L)}
    conn.register_kv_caches(caches)
    perm = np.random.default_rng(4).permutation(NBLK)
    bt = [perm[0:40].tolist(), perm[40:80].tolist(), perm[80:120].tolist()]
    ctx = SimpleNamespace(no_compile_layers={}, virtual_engine=0)

    def rows(kv, blocks, lo, hi):  # [n, H, 2D] bits of positions [lo, hi)
        pos = np.arange(lo, hi)
        blk = np.asarray(blocks)[pos // BS]
        return kv.cpu().view(torch.int16).numpy().view(np.uint16)[blk, pos % BS]

    def step(meta, save=True):
        conn.bind_connector_metadata(meta)
        conn.start_load_kv(ctx)
        for name in caches:
            conn.wait_for_layer_load(name)
        if save:
            for name, kv in caches.items():
                conn.save_kv_layer(name, kv, None)
        conn.wait_for_save()
        conn.clear_connector_metadata()
        torch.cuda.synchronize()

    # turn 0: positions [0, 600) computed and saved as generation 0
    step(C.ShiftConnectorMetadata(saves=[C._Save("s", 0, 600, bt[0], BS, 0)]))
    gen0 = {n: rows(kv, bt[0], 0, 600) for n, kv in caches.items()}
    # turn 1: [0, 100) replaced by 137 fresh tokens (generation 1); [100, 600) -> +37
    step(C.ShiftConnectorMetadata(
        loads=[C._Load("s", 100, 37, 137, 500, bt[1], BS, 0)],
        saves=[C._Save("s", 0, 137, bt[1], BS, 1)],
        releases=[("s", 0, 0, 100)]))
    gen1 = {n: rows(kv, bt[1], 0, 137) for n, kv in caches.items()}
    # turn 2: [0, 50) deleted: generation 1's [50, 137) -> [0, 87) by -50 and
    # generation 0's [100, 600) -> [87, 587): one rotation of -13 from turn 0's bytes
    step(C.ShiftConnectorMetadata(
        loads=[C._Load("s", 50, -50, 0, 87, bt[2], BS, 1),
               C._Load("s", 100, -13, 87, 500, bt[2], BS, 0)],
        releases=[("s", 1, 0, 50)]), save=False)

    inv = conn._inv_freq.numpy()
    t50, t13 = reference_tables([-50, -13], inv, cuda)
    for name, kv in caches.items():
        got = rows(kv, bt[2], 0, 587)
        want1 = gen1[name][50:137]
        want0 = gen0[name][100:600]
        assert np.array_equal(got[:87, :, D:], want1[..., D:])
        assert np.array_equal(got[:87, :, :D], O.shift_k_bits(want1[..., :D], t50, O.BF16))
        assert np.array_equal(got[87:, :, D:], want0[..., D:])
        assert np.array_equal(got[87:, :, :D], O.shift_k_bits(want0[..., :D], t13, O.BF16))
    st = conn._store
    assert st.locate("s", 0, 0, 100, count=False) is None
    assert st.locate("s", 1, 0, 50, count=False) is None
    assert st.locate("s", 0, 100, 500, count=False) is not None


def test_extent_mode_worker_splits_loads_and_saves_by_extent():
    """Worker-side translation (no GPU): a load spanning two extents of a
    generation becomes two jobs with their own store rows; a save gets the rows
    the scheduler allocated for the same call."""
    conn = C.MarathonShiftConnector(fake_config({"store_tokens": 8192, "store_mode": "extents",
                                                 "store_device": "cpu"}),
                                    KVConnectorRole.WORKER, None)
    st = conn._store
    st.save_extent("s", 0, 0, 100)
    st.save_extent("s", 1, 0, 50)  # another generation takes the next rows
    st.save_extent("s", 0, 100, 60)  # generation 0 continues elsewhere
    jobs, lost = conn._extent_load_jobs([C._Load("s", 40, 12, 52, 100, [0, 1, 2], BS, 0)])
    assert [(j.src_start, j.length, j.store_start, j.dst_start, j.delta) for j in jobs] == \
        [(40, 60, 40, 52, 12), (100, 40, 150, 112, 12)] and lost == []
    saves = conn._extent_save_jobs(C._Save("s", 160, 30, [0, 1, 2], BS, 0))
    assert [(j.dst_start, j.length, j.store_start) for j in saves] == [(160, 30, 210)]
    unknown = C._Load("s", 0, 0, 0, 10, [0], BS, 7)  # a generation the store never held
    assert conn._extent_load_jobs([unknown]) == ([], [unknown])


# ------------------------------------------------- failures: decline, never guess
def test_failed_save_is_forgotten_by_worker_and_scheduler_mirror():
    """A save the kernel refused truncates the session on the worker; the worker
    metadata carries the truncation to the scheduler's mirror, whose next plan
    declines the span instead of loading rows that were never written."""
    sched = scheduler()
    worker = C.MarathonShiftConnector(fake_config({"store_tokens": 65536, "store_device": "cpu"}),
                                      KVConnectorRole.WORKER, None)
    for st in (sched._store, worker._store):
        assert st.reserve("s", 0, 600)
    save = C._Save("s", 0, 600, list(range(40)), BS)
    worker._saves_failed([save], 1)  # the step's status word had MSHIFT_EBIT_SLOT
    assert worker.save_failures == 1 and not worker._store.covers("s", 64, 16)
    wmeta = worker.build_connector_worker_meta()
    assert isinstance(wmeta, C.ShiftWorkerMetadata) and wmeta.truncate == [("s", 0)]
    assert worker.build_connector_worker_meta() is None  # reported once
    sched.update_connector_output(SimpleNamespace(kv_connector_worker_meta=wmeta))
    r = request("r1", {"session": "s", "load": {"dst_start": 64, "dst_end": 600, "delta": 8}},
                700)
    sched.on_new_request(r)
    assert sched.get_num_new_matched_tokens(r, 64) == (0, False)
    # a later save that would leave a hole above the truncation is refused on both sides
    assert not sched._store.reserve("s", 600, 10) and not worker._store.reserve("s", 600, 10)


def test_worker_metadata_aggregates_ranks():
    a = C.ShiftWorkerMetadata(truncate=[("s", 0)])
    b = C.ShiftWorkerMetadata(release=[("t", 1, 0, 16)])
    ab = a.aggregate(b)
    assert ab.truncate == [("s", 0)] and ab.release == [("t", 1, 0, 16)] and ab
    assert not C.ShiftWorkerMetadata()


def test_failed_extent_save_releases_that_generation():
    sched = scheduler({"store_tokens": 8192, "store_mode": "extents"})
    worker = C.MarathonShiftConnector(fake_config({"store_tokens": 8192, "store_mode": "extents",
                                                   "store_device": "cpu"}),
                                      KVConnectorRole.WORKER, None)
    for st in (sched._store, worker._store):
        assert st.save_extent("s", 0, 0, 300)
    worker._saves_failed([C._Save("s", 0, 300, list(range(19)), BS, 0)], 2)
    wmeta = worker.build_connector_worker_meta()
    assert wmeta.release == [("s", 0, 0, 300)]
    sched.update_connector_output(SimpleNamespace(kv_connector_worker_meta=wmeta))
    for st in (sched._store, worker._store):
        assert st.locate("s", 0, 0, 300, count=False) is None


def test_load_errors_name_the_destination_blocks():
    from marathon_b200.worker import LoadJob

    conn = C.MarathonShiftConnector(fake_config({"store_tokens": 8192, "store_device": "cpu"}),
                                    KVConnectorRole.WORKER, None)
    table = list(range(100, 140))
    conn._note_load_errors([LoadJob("s", 0, 0, 32, 48, block_ids=table),  # blocks 2..4
                            LoadJob("s", 0, 0, 100, 1, block_ids=table)])  # block 6
    assert conn.get_block_ids_with_load_errors() == {102, 103, 104, 106}
    assert conn.get_block_ids_with_load_errors() == set()


def test_registration_runs_warmup(monkeypatch):
    seen = []
    monkeypatch.setattr(C, "warmup", lambda kv, bs, hnd, **kw: seen.append((bs, hnd, kw)))
    conn = C.MarathonShiftConnector(fake_config({"store_tokens": 8192}),
                                    KVConnectorRole.WORKER, None)
    conn.register_kv_caches({"l0": torch.zeros(4, BS, 2, 256, dtype=torch.bfloat16)})
    assert seen == [(BS, False, {"rotary": 128, "layout": "nhd", "fp8": False})]


def test_ulp_matches_the_dtype_spacing():
    x = torch.tensor([1.0, 1.5, 2.0, 3.0, -0.75, 0.0, 1e-40, 2.0**-126], dtype=torch.float32)
    want = [2.0**-7, 2.0**-7, 2.0**-6, 2.0**-6, 2.0**-8, 2.0**-133, 2.0**-133, 2.0**-133]
    assert C.ulp(x, torch.bfloat16).tolist() == want
    assert C.ulp(torch.tensor([1.0]), torch.float16).tolist() == [2.0**-10]
    # the next bf16 value above x is exactly one ulp away
    for v in (1.0, 3.0, 1000.0, 2.0**-120):
        t = torch.tensor([v], dtype=torch.bfloat16)
        nxt = t.view(torch.int16) + 1
        assert float(nxt.view(torch.bfloat16)) - v == float(C.ulp(t.float(), torch.bfloat16))


def _worker_with_caches(cuda, extra=None, L=3, NBLK=96, H=8, D=128, seed=7):
    cfg = {"store_tokens": 8192, **(extra or {})}
    conn = C.MarathonShiftConnector(fake_config(cfg), KVConnectorRole.WORKER, None)
    g = torch.Generator().manual_seed(seed)
    caches = {f"model.layers.{i}.self_attn.attn":
              torch.randn(NBLK, BS, H, 2 * D, generator=g).to(torch.bfloat16).to(cuda)
              for i in range(L)}
    conn.register_kv_caches(caches)
    return conn, caches


def _save_step(conn, caches, saves):
    conn.bind_connector_metadata(C.ShiftConnectorMetadata(saves=saves))
    for name, kv in caches.items():
        conn.save_kv_layer(name, kv, None)
    conn.wait_for_save()
    conn.clear_connector_metadata()


@pytest.mark.gpu
@pytest.mark.parametrize("batch_save", [False, True])
def test_refused_save_makes_the_next_edit_turn_recompute(cuda, batch_save):
    """A save whose block table holds an out-of-range block id: the kernel skips
    those tokens and flags them; the session is truncated on the worker and,
    through the worker metadata, in the scheduler's mirror, so the next edit
    turn recomputes instead of loading the stale rows.  The control run with a
    valid table loads."""
    outcomes = {}
    for bad in (False, True):
        sched = scheduler({"store_tokens": 8192})
        conn, caches = _worker_with_caches(cuda, {"batch_save": batch_save})
        r0 = request("r0", {"session": "s", "save": True}, 600)
        sched.on_new_request(r0)
        assert sched.get_num_new_matched_tokens(r0, 0) == (0, False)
        blocks0 = list(range(40))
        if bad:
            blocks0[20] = 96 + 5  # past the last block of the cache
        meta = sched.build_connector_meta(sched_output([new_req("r0", blocks0, 0)],
                                                       scheduled={"r0": 600}))
        sched.request_finished(r0, blocks0)
        conn._store.reserve("s", 0, 600)  # the worker mirrors the scheduler's reserve
        _save_step(conn, caches, meta.saves)
        torch.cuda.synchronize()
        wmeta = conn.build_connector_worker_meta()
        sched.update_connector_output(SimpleNamespace(kv_connector_worker_meta=wmeta))
        r1 = request("r1", {"session": "s", "load": {"dst_start": 64, "dst_end": 600,
                                                     "delta": 24}}, 700)
        sched.on_new_request(r1)
        outcomes[bad] = (sched.get_num_new_matched_tokens(r1, 64)[0], conn.save_failures,
                         wmeta)
    n_ok, fails_ok, meta_ok = outcomes[False]
    n_bad, fails_bad, meta_bad = outcomes[True]
    assert n_ok == 592 - 64 and fails_ok == 0 and meta_ok is None
    assert n_bad == 0 and fails_bad == 1 and meta_bad.truncate == [("s", 0)]


@pytest.mark.gpu
def test_refused_load_reports_its_blocks(cuda):
    """A queued load whose block table points past the cache: the status read at
    wait_for_save names the load's destination blocks for vLLM to recompute."""
    conn, caches = _worker_with_caches(cuda)
    assert conn._store.reserve("s", 0, 600)
    _save_step(conn, caches, [C._Save("s", 0, 600, list(range(40)), BS)])
    bt = list(range(40, 80))
    bt[10] = 96 + 1
    conn.bind_connector_metadata(C.ShiftConnectorMetadata(
        loads=[C._Load("s", 64, 16, 80, 512, bt, BS)]))
    conn.start_load_kv(forward_context())
    conn.wait_for_save()
    conn.clear_connector_metadata()
    assert conn.get_block_ids_with_load_errors() == set(bt[80 // BS : (80 + 512) // BS])


@pytest.mark.gpu
def test_verify_load_passes_a_correct_load_and_reports_a_planted_mismatch(cuda, monkeypatch):
    """``MARATHON_VERIFY_LOAD``: every loaded layer is read back and held to the
    north-star bar against torch's fp32 rotation with the reference's tables.
    A correct load passes.  Then the mistake is planted in the checker's own
    input on the CPU (the inverse frequencies it rotates with are perturbed),
    and the check must report the mismatch and the load's blocks."""
    monkeypatch.setattr(C, "VERIFY_LOAD", True)
    conn, caches = _worker_with_caches(cuda)
    assert conn._store.reserve("s", 0, 600)
    _save_step(conn, caches, [C._Save("s", 0, 600, list(range(40)), BS)])
    bt = list(range(40, 80))

    def load(delta):
        conn.bind_connector_metadata(C.ShiftConnectorMetadata(
            loads=[C._Load("s", 64, delta, 64 + delta, 512, bt, BS)]))
        conn.start_load_kv(forward_context())
        conn.wait_for_save()
        conn.clear_connector_metadata()

    load(16)
    assert conn.verify_mismatches == 0 and conn.get_block_ids_with_load_errors() == set()
    monkeypatch.setattr(conn, "_inv_freq", conn._inv_freq * 1.001)
    load(32)
    assert conn.verify_mismatches == 1
    assert conn.get_block_ids_with_load_errors() == set(bt[96 // BS : (96 + 512) // BS])


@pytest.mark.gpu
def test_registration_rejects_a_geometry_no_kernel_serves(cuda):
    conn = C.MarathonShiftConnector(fake_config({"store_tokens": 8192}, head_dim=96),
                                    KVConnectorRole.WORKER, None)
    from marathon_b200.shift_kernels import ShiftError

    with pytest.raises(ShiftError, match="no kernel"):
        conn.register_kv_caches({"l0": torch.zeros(8, BS, 2, 192, dtype=torch.bfloat16,
                                                   device=cuda)})
