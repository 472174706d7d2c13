"""Store bookkeeping on CPU: the reference's store cases, run against marathon_b200.

Each case restates one of the reference's store tests
(``tests/test_shift_store.py`` of acrosley/marathon, cited per test); KV is
faked with small CPU tensors because ``write``/``read`` are plain tensor
copies and views whatever device the store is on.
"""

from __future__ import annotations

import pytest
import torch

from marathon_b200.shift_store import (
    SLAB,
    LoadDecision,
    SessionTable,
    ShiftStore,
    churn_tokens,
    plan_load,
    plan_save,
    slots,
)


def _kv(n: int, value: float, heads: int = 2, dim: int = 4) -> torch.Tensor:
    return torch.full((n, heads, dim), value)


def store(**kw) -> ShiftStore:
    kw.setdefault("device", "cpu")
    return ShiftStore(**kw)


def test_slots_map_positions_through_the_block_table():  # :24-27
    assert slots([7, 3], 2, 6, block_size=4).tolist() == [30, 31, 12, 13]


def test_session_table_refuses_a_second_in_flight_writer():  # :33-41
    t = SessionTable()
    assert t.acquire("r1", "s")
    assert not t.acquire("r2", "s")
    assert t.session_of("r2") is None and t.conflicts == 1
    t.release("r1")
    assert t.acquire("r2", "s") and t.session_of("r2") == "s"


def test_session_table_reacquire_and_unknown_release():  # :44-56
    t = SessionTable()
    assert t.acquire("r1", "s") and t.acquire("r1", "s") and t.conflicts == 0
    t.release("nobody")
    assert t.session_of("r1") == "s" and len(t) == 1


def test_append_only_saves_extend_the_filled_span():  # :62-67
    st = store(slab=1024, budget_tokens=4096)
    assert st.reserve("a", 0, 100) and st.reserve("a", 100, 50)
    assert st.covers("a", 0, 150) and not st.covers("a", 0, 151)


def test_a_save_that_would_leave_a_hole_is_refused():  # :70-75
    st = store(slab=1024, budget_tokens=4096)
    st.reserve("a", 0, 100)
    assert not st.reserve("a", 200, 10)
    assert st.covers("a", 0, 100) and st.refusals == 1


def test_an_edit_truncates_everything_above_it():  # :78-84
    st = store(slab=1024, budget_tokens=4096)
    st.reserve("a", 0, 500)
    assert st.reserve("a", 200, 60)
    assert st.covers("a", 0, 260) and not st.covers("a", 0, 300)


def test_a_span_larger_than_the_budget_is_refused():  # :87-90
    st = store(slab=1024, budget_tokens=1024)
    assert not st.reserve("a", 0, 2000) and not st.covers("a", 0, 1)


def test_reserve_is_idempotent():  # :93-97
    st = store(slab=1024, budget_tokens=4096)
    for _ in range(5):
        assert st.reserve("a", 0, 300)
    assert st.stats()["sessions"] == {"a": 300}


def test_write_read_round_trip_and_session_isolation():  # :103-113
    st = store(slab=1024, budget_tokens=4096)
    st.reserve("a", 0, 8)
    st.reserve("b", 0, 8)
    st.write("a", "layer0", 0, _kv(8, 1.0))
    st.write("b", "layer0", 0, _kv(8, 2.0))
    assert torch.equal(st.read("a", "layer0", 0, 8), _kv(8, 1.0))
    assert torch.equal(st.read("b", "layer0", 0, 8), _kv(8, 2.0))
    assert st.read("a", "layer1", 0, 8) is None
    assert st.read("nobody", "layer0", 0, 8) is None


def test_read_past_the_filled_span_returns_none():  # :116-120
    st = store(slab=1024, budget_tokens=4096)
    st.reserve("a", 0, 8)
    st.write("a", "layer0", 0, _kv(8, 1.0))
    assert st.read("a", "layer0", 4, 8) is None


def test_growth_preserves_already_stored_kv():  # :123-130
    st = store(slab=1024, budget_tokens=8192)
    st.reserve("a", 0, 100)
    st.write("a", "layer0", 0, _kv(100, 3.0))
    st.reserve("a", 100, 2000)
    st.write("a", "layer0", 100, _kv(2000, 4.0))
    assert torch.equal(st.read("a", "layer0", 0, 100), _kv(100, 3.0))
    assert torch.equal(st.read("a", "layer0", 100, 2000), _kv(2000, 4.0))


def test_lru_evicts_the_least_recently_used_session():  # :136-145
    st = store(slab=1024, budget_tokens=3072)
    for s in "abc":
        st.reserve(s, 0, 1000)
    st.covers("a", 0, 1000)
    st.reserve("c", 1000, 500)
    assert st.stats()["evictions"] == 1
    assert set(st.stats()["sessions"]) == {"a", "c"}
    assert not st.covers("b", 0, 10)


def test_eviction_never_takes_the_session_being_written():  # :148-154
    st = store(slab=1024, budget_tokens=2048)
    st.reserve("a", 0, 1000)
    st.reserve("b", 0, 1000)
    st.reserve("b", 1000, 1000)
    assert set(st.stats()["sessions"]) == {"b"} and st.covers("b", 0, 2000)


def test_an_evicted_session_is_a_miss_not_a_wrong_load():  # :157-164
    st = store(slab=1024, budget_tokens=2048)
    st.reserve("a", 0, 1000)
    st.write("a", "layer0", 0, _kv(1000, 9.0))
    st.reserve("b", 0, 2000)
    assert not st.covers("a", 0, 1000)
    assert st.read("a", "layer0", 0, 1000) is None and st.misses == 1


def test_bookkeeping_only_mode_tracks_positions_without_tensors():  # :167-175
    sched = store(slab=1024, budget_tokens=4096, allocate=False)
    worker = store(slab=1024, budget_tokens=4096)
    for start, n in ((0, 500), (500, 500), (200, 100)):
        assert sched.reserve("a", start, n) == worker.reserve("a", start, n)
    sched.write("a", "layer0", 0, _kv(8, 1.0))
    assert sched.read("a", "layer0", 0, 8) is None
    assert sched.stats()["sessions"] == worker.stats()["sessions"] == {"a": 300}


def test_stats_reports_tokens_per_session():  # :178-186
    st = store(slab=1024, budget_tokens=4096)
    st.reserve("a", 0, 300)
    st.reserve("b", 0, 700)
    st.write("b", "layer0", 0, _kv(700, 1.0))
    s = st.stats()
    assert s["sessions"] == {"a": 300, "b": 700}
    assert s["saved_token_layers"] == 700 and s["budget_tokens"] == 4096


def test_the_first_save_may_start_above_zero():  # :189-198
    st = store(slab=1024, budget_tokens=4096)
    assert st.reserve("a", 16, 600) and st.reserve("a", 616, 600)
    assert st.covers("a", 616, 600) and st.covers("a", 16, 1200)
    assert not st.covers("a", 0, 1216)
    assert st.read("a", "layer0", 0, 16) is None


# ----------------------------------------------- presizing (test_paged_depth.py:455-497)
def _count_grows(monkeypatch):
    grows = []
    original = ShiftStore._grow

    def counted(self, session, entry, want):
        grows.append((session, entry.capacity, want))
        return original(self, session, entry, want)

    monkeypatch.setattr(ShiftStore, "_grow", counted)
    return grows


def test_presizing_allocates_once(monkeypatch):
    st = store(budget_tokens=24576, session_cap=8192)
    grows = _count_grows(monkeypatch)
    for hi in range(256, 8192, 256):
        assert st.reserve("s", 0, hi)
    assert len(grows) == 1 and st._sessions["s"].capacity == 8192 and st.evictions == 0


def test_presizing_is_a_floor_not_a_ceiling():
    st = store(budget_tokens=24576, session_cap=4096)
    assert st.reserve("s", 0, 4000) and st._sessions["s"].capacity == 4096
    assert st.reserve("s", 0, 9000) and st._sessions["s"].capacity >= 9000
    assert st.covers("s", 0, 9000)


def test_presizing_off_by_default_keeps_geometric_growth():
    st = store(budget_tokens=24576)
    assert st.session_cap == 0 and st.reserve("s", 0, 100)
    assert st._sessions["s"].capacity == SLAB


def test_the_flat_store_truncates_where_a_remap_would_need_bytes():  # test_paged_depth.py:553-563
    st = store(budget_tokens=8192, allocate=False)
    assert st.reserve("s", 0, 1000) and st.covers("s", 900, 100)
    assert st.reserve("s", 200, 50)
    assert not st.covers("s", 900, 100)


# ------------------------------------------------------------ plan_load / plan_save
def test_plan_load_aligns_to_blocks_and_leaves_a_token():
    st = store(budget_tokens=8192)
    st.reserve("s", 0, 2000)
    d, why = plan_load(st, "s", {"dst_start": 300, "dst_end": 1900, "delta": 20}, 304, 1000, 16)
    assert why == "ok" and d == LoadDecision(304, 992, 20) and d.src_start == 284


@pytest.mark.parametrize("args,reason", [
    ((None, {"dst_start": 0, "dst_end": 10, "delta": 1}, 0, 100), "no session"),
    (("s", None, 0, 100), "no session"),
    (("s", {"dst_start": 64, "dst_end": 640, "delta": 1}, 32, 700), "local hit"),
    (("s", {"dst_start": 0, "dst_end": 10, "delta": 1}, 0, 100), "nothing left"),
    (("s", {"dst_start": 0, "dst_end": 640, "delta": -5000}, 0, 700), "no longer holds"),
])
def test_plan_load_declines(args, reason):
    st = store(budget_tokens=8192)
    st.reserve("s", 0, 2000)
    session, req, computed, n_prompt = args
    d, why = plan_load(st, session, req, computed, n_prompt, 16)
    assert d is None and reason in why


def test_plan_save_full_widens_and_refusal_returns_none():
    st = store(budget_tokens=8192)
    assert plan_save(st, "s", "full", 100, 300) == (0, 300)
    assert plan_save(st, "s", True, 300, 310) == (300, 310)
    assert plan_save(st, "s", True, 400, 410) is None  # hole
    assert plan_save(st, None, True, 0, 10) is None
    assert plan_save(st, "s", False, 0, 10) is None


def test_churn_tokens():
    assert churn_tokens([]) == (0, 0)
    assert churn_tokens([{"dst_start": 100, "dst_end": 400}]) == (100, 300)
    two = [{"dst_start": 0, "dst_end": 50}, {"dst_start": 80, "dst_end": 200}]
    assert churn_tokens(two) == (30, 170)


def test_adopt_and_view_expose_buffers():
    st = store(budget_tokens=8192)
    bufs = {"l0": torch.zeros(64, 2, 8), "l1": torch.zeros(64, 2, 8)}
    st.adopt("s", bufs, 0, 64)
    assert st.covers("s", 0, 64)
    v = st.view(["s", "t"], ["l0", "l1", "l2"])
    assert v.ptrs[0, 0] == bufs["l0"].data_ptr() and v.ptrs[0, 2] == 0 and v.ptrs[1, 0] == 0
    assert v.caps.tolist() == [64, 0] and (v.st_tok, v.st_head) == (16, 8)
    assert st.loadable("s", ["l0", "l1"], 0, 64) is None
    assert st.loadable("s", ["l0", "l2"], 0, 64) == "l2"
    assert st.loadable("s", ["l0"], 10, 60) == "l0"
