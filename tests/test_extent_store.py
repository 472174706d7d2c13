"""The generation-tagged interval store and its address book, on the CPU.

The fingerprint model of the reference's paged-depth harness: the "keys" of a
token computed at position ``p`` are ``(token, p)`` and a re-rotation by
``delta`` turns them into ``(token, p + delta)``, exactly.  A load is right
iff the bytes it lands at logical position ``q`` read ``(token at q, q)``.
Turn after turn of front, middle and tail edits, with no span ever re-saved,
every load must come back right and must read the rows of the generation
that first computed the token -- the property the flat store cannot give
(``tests/test_shift_store.py`` pins the truncation that breaks it).
"""

from __future__ import annotations

import numpy as np
import pytest

from marathon_b200.extent_store import AddressBook, ExtentStore


# ------------------------------------------------------------------ store
def test_save_is_idempotent_and_extends_in_place():
    st = ExtentStore(4096, device="cpu", allocate=False, slab=256)
    a = st.save_extent("s", 0, 0, 100)
    assert a == [(0, 100, 0)]
    assert st.save_extent("s", 0, 0, 100) == a  # same generation, same positions
    b = st.save_extent("s", 0, 100, 50)  # decode steps append
    assert b == [(100, 50, 100)]
    assert st.locate("s", 0, 0, 150) == [(0, 150, 0)]
    assert len(st._sessions["s"].extents[0]) == 1  # one extent, grown in place


def test_generations_never_share_rows():
    st = ExtentStore(4096, device="cpu", allocate=False, slab=256)
    st.save_extent("s", 0, 0, 300)
    fresh = st.save_extent("s", 1, 200, 64)  # same positions, a later generation
    rows0 = {r for _, n, r0 in st.locate("s", 0, 0, 300) for r in range(r0, r0 + n)}
    rows1 = {r for _, n, r0 in fresh for r in range(r0, r0 + n)}
    assert rows0.isdisjoint(rows1)
    assert st.locate("s", 0, 200, 64) is not None  # generation 0 still intact


def test_partial_overlap_reuses_held_rows_and_allocates_the_rest():
    st = ExtentStore(4096, device="cpu", allocate=False, slab=256)
    st.save_extent("s", 3, 100, 50)
    out = st.save_extent("s", 3, 80, 100)  # [80, 100) new, [100, 150) held, [150, 180) new
    assert [(p, n) for p, n, _ in out] == [(80, 20), (100, 50), (150, 30)]
    assert out[1][2] == st.locate("s", 3, 100, 1)[0][2]
    assert st.locate("s", 3, 80, 100) is not None


def test_release_frees_rows_for_reuse_and_splits_extents():
    st = ExtentStore(1024, device="cpu", allocate=False, slab=256)
    st.save_extent("s", 0, 0, 200)
    assert st.release("s", 0, 50, 100) == 100
    assert st.locate("s", 0, 0, 50) is not None and st.locate("s", 0, 150, 50) is not None
    assert st.locate("s", 0, 60, 10) is None
    out = st.save_extent("s", 1, 0, 100)  # fits in the freed hole, no growth
    assert st.capacity("s") == 256 and out[0][2] == 50


def test_growth_keeps_rows_and_budget_evicts_lru():
    st = ExtentStore(1024, device="cpu", allocate=False, slab=256)
    st.save_extent("a", 0, 0, 400)
    st.save_extent("b", 0, 0, 300)  # a: 512, b: 512 -> full budget
    assert st.used == 1024
    st.locate("a", 0, 0, 10)  # a becomes most recent
    st.save_extent("c", 0, 0, 100)  # needs room: evicts b, the least recent
    assert "b" not in st._sessions and st.evictions == 1
    assert st.locate("a", 0, 0, 400) == [(0, 400, 0)]
    assert st.save_extent("d", 0, 0, 2048) == [] and st.refusals >= 1


def test_loadable_checks_allocated_rows():
    st = ExtentStore(1024, device="cpu", allocate=True, slab=256)
    st.save_extent("s", 0, 0, 100)
    st._sessions["s"].layers = {"l0": None}
    assert st.loadable("s", ["l0"], 0, 100) is None
    assert st.loadable("s", ["l0"], 50, 100) == "l0"  # rows 100..149 are free
    assert st.loadable("s", ["l1"], 0, 10) == "l1"


# ------------------------------------------------------------ address book
def test_loads_carry_generation_and_rotate_from_pos0():
    bk = AddressBook()
    assert bk.after_turn([], 1000, 0) == []
    segs = [{"dst_start": 0, "dst_end": 200, "delta": 0},
            {"dst_start": 264, "dst_end": 1024, "delta": 24}]
    assert bk.loads(segs)[1] == {"dst_start": 264, "dst_end": 1024, "delta": 24, "gen": 0,
                                 "src_start": 240}
    dead = bk.after_turn(segs, 1100, 1)
    assert dead == [(0, 200, 40)]  # the edited span [200, 240) of generation 0
    # next turn moves the tail again: one rotation from generation 0, offsets add
    segs2 = [{"dst_start": 0, "dst_end": 1000, "delta": -100}]
    loads = bk.loads(segs2)
    assert [(ld["gen"], ld["src_start"], ld["delta"]) for ld in loads] == \
        [(0, 100, -100), (1, 200, -100), (0, 240, -76), (1, 1024, -100)]


class _Harness:
    """A session of edits driven through the store and the address book."""

    def __init__(self, seed: int, budget: int = 1 << 16) -> None:
        self.rng = np.random.default_rng(seed)
        self.store = ExtentStore(budget, device="cpu", allocate=False, slab=512)
        self.book = AddressBook()
        self.rows: dict[int, tuple[int, int]] = {}  # store row -> (token, pos computed at)
        self.tokens: list[int] = []
        self.next_token = 0
        self.gen = 0
        self.first_gen: dict[int, int] = {}  # token -> generation that computed it
        self.loads_checked = 0

    def _fresh(self, n: int) -> list[int]:
        out = list(range(self.next_token, self.next_token + n))
        self.next_token += n
        return out

    def turn(self, kind: str) -> None:
        old = self.tokens
        n = len(old)
        if not old:
            new, segs = self._fresh(int(self.rng.integers(200, 600))), []
        else:
            a = 0 if kind == "front" else int(self.rng.integers(0, n))
            if kind == "tail":
                a = max(0, n - int(self.rng.integers(1, 30)))
            b = min(n, a + int(self.rng.integers(1, 60)))
            ins = self._fresh(int(self.rng.integers(0, 80)))
            new = old[:a] + ins + old[b:] + self._fresh(int(self.rng.integers(1, 40)))
            segs = []
            if a > 0:
                segs.append({"dst_start": 0, "dst_end": a, "delta": 0})
            if b < n:
                d = len(ins) - (b - a)
                segs.append({"dst_start": b + d, "dst_end": n + d, "delta": d})
        gen = self.gen
        self.gen += 1
        # loads first (against the view before the turn), as the server sends them
        loaded = set()
        for ld in self.book.loads(segs):
            q_lo, q_hi = ld["dst_start"], ld["dst_end"]
            where = self.store.locate("s", ld["gen"], ld["src_start"], q_hi - q_lo)
            assert where is not None, ("miss", ld)
            q = q_lo
            for _, cnt, row in where:
                for r in range(row, row + cnt):
                    tok, p = self.rows[r]
                    assert (tok, p + ld["delta"]) == (new[q], q), ("wrong bytes", ld, q)
                    assert self.first_gen[tok] == ld["gen"]
                    loaded.add(q)
                    q += 1
            self.loads_checked += 1
        for g, p0, cnt in self.book.after_turn(segs, len(new), gen):
            self.store.release("s", g, p0, cnt)
        # the engine computes everything not loaded; the connector saves it
        q = 0
        while q < len(new):
            if q in loaded:
                q += 1
                continue
            r = q
            while r < len(new) and r not in loaded:
                r += 1
            for p0, cnt, row in self.store.save_extent("s", gen, q, r - q):
                for i in range(cnt):
                    tok = new[p0 + i]
                    self.rows[row + i] = (tok, p0 + i)
                    self.first_gen.setdefault(tok, gen)
            q = r
        self.tokens = new


@pytest.mark.parametrize("seed", range(6))
def test_many_turns_of_edits_always_load_generation_zero_bytes(seed):
    h = _Harness(seed)
    kinds = ["front", "mid", "tail"]
    for t in range(40):
        h.turn(kinds[(t + seed) % 3])
    assert h.loads_checked > 30
    # rows in use equal the view: every dead extent was released
    used = h.store._sessions["s"].used_rows()
    assert used == len(h.tokens)


def test_thirty_front_edits_keep_every_coordinate_exact():
    h = _Harness(11)
    for _ in range(31):
        h.turn("front")
    assert h.loads_checked >= 30


def test_scheduler_mirror_and_worker_store_stay_identical_under_eviction():
    """The two copies see the same operations in the same order (the scheduler
    checks coverage and plans saves; the worker applies releases, loads and
    saves) and so allocate identical rows, evictions included."""
    rng = np.random.default_rng(5)
    sched = ExtentStore(6000, device="cpu", allocate=False, slab=512)
    work = ExtentStore(6000, device="cpu", allocate=False, slab=512)
    held: dict[str, list[tuple[int, int, int]]] = {}
    for step in range(300):
        s = f"s{int(rng.integers(0, 6))}"
        gen = step
        # a load of something this session saved earlier (if still held)
        if held.get(s):
            g, p0, n = held[s][int(rng.integers(0, len(held[s])))]
            a = sched.locate(s, g, p0, n)  # scheduler coverage check (touches)
            if a is not None:
                b = work.locate(s, g, p0, n, count=False)
                assert a == b
                work.mark_loaded(s, ["l0"], n)  # the worker's touch for the load
        # a release of one old extent, then this step's save
        if held.get(s) and rng.random() < 0.4:
            g, p0, n = held[s].pop(0)
            assert sched.release(s, g, p0, n) == work.release(s, g, p0, n)
        p0, n = int(rng.integers(0, 4000)), int(rng.integers(1, 800))
        a = sched.save_extent(s, gen, p0, n)
        b = work.save_extent(s, gen, p0, n)
        assert a == b
        if a:
            held.setdefault(s, []).append((gen, p0, n))
        for name in list(held):
            if name not in sched._sessions:
                held.pop(name)
        assert list(sched._sessions) == list(work._sessions)
        for name in sched._sessions:
            x, y = sched._sessions[name], work._sessions[name]
            assert x.capacity == y.capacity and x.free == y.free
            assert {g: [(e.pos0, e.n, e.row) for e in v] for g, v in x.extents.items()} == \
                {g: [(e.pos0, e.n, e.row) for e in v] for g, v in y.extents.items()}
    assert sched.evictions > 0 and sched.evictions == work.evictions
