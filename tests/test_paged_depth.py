"""Coordinates through many consecutive edit turns, on CPU, with KV modelled as token ids.

The reference pins "every position holds its own token" through 30 front edits
with negative deltas (``tests/test_paged_depth.py:200-238`` of acrosley/marathon).
Its harness drives the full server; here a small turn driver produces the same
shape of plans (a front demotion that shrinks the view, a mid edit that grows
it, appends) and a fake paged engine applies the connector's decisions —
``plan_load`` / ``plan_save`` / ``ShiftStore`` from ``marathon_b200`` — with
a block-granular prefix cache and one save per scheduler step, decode steps
included.  Because "KV" is the token id, any coordinate error is a visible
corruption; rotation is exact by construction and not what is tested here.
"""

from __future__ import annotations

import torch

from marathon_b200.shift_store import ShiftStore, plan_load, plan_save, slots

BS = 16


class Engine:
    """Paged cache (slot -> token id), block prefix cache, per-step saves."""

    def __init__(self, budget=1 << 20):
        self.store = ShiftStore(budget, device="cpu")
        self.cache: list[int] = []
        self.prefix: dict[tuple, int] = {}
        self.corrupt: list[tuple] = []
        self.declined: list[str] = []
        self.loaded = 0
        self.refused = 0
        self.turn = 0

    def _block(self) -> int:
        self.cache.extend([0] * BS)
        return len(self.cache) // BS - 1

    def _table(self, ids):
        blocks, hit, broken = [], 0, False
        for k in range(-(-len(ids) // BS)):
            key = tuple(ids[: (k + 1) * BS])
            b = None if broken else self.prefix.get(key)
            if b is not None and (k + 1) * BS <= len(ids):
                blocks.append(b)
                hit = (k + 1) * BS
            else:
                broken = True
                blocks.append(self._block())
        return blocks, hit

    def _put(self, blocks, lo, hi, vals):
        for s, v in zip(slots(blocks, lo, hi, BS).tolist(), vals, strict=True):
            self.cache[s] = v

    def _get(self, blocks, lo, hi):
        return [self.cache[s] for s in slots(blocks, lo, hi, BS).tolist()]

    def _step(self, params, blocks, lo, hi, session):
        w = plan_save(self.store, session, params.get("save"), lo, hi)
        if w is None:
            if params.get("save") and hi > lo:
                self.refused += 1
            return
        if params.get("save") == "full":
            params["save"] = True
        a, b = w
        vals = torch.tensor(self._get(blocks, a, b), dtype=torch.float32).reshape(-1, 1, 1)
        self.store.write(session, "L0", a, vals)

    def generate(self, ids, session, load=None, save=True, decode=3):
        blocks, computed = self._table(ids)
        params = {"save": save}
        d, why = plan_load(self.store, session, load, computed, len(ids), BS)
        if load and d is None:
            self.declined.append(f"turn {self.turn}: {why}")
        if d is not None:
            rows = self.store.read(session, "L0", d.src_start, d.hi - d.lo)
            assert rows is not None
            self._put(blocks, d.lo, d.hi, [int(v) for v in rows[:, 0, 0].tolist()])
            self.loaded += d.hi - d.lo
            computed = d.hi
        self._put(blocks, computed, len(ids), ids[computed:])
        for pos, got in enumerate(self._get(blocks, 0, len(ids))):
            if got != ids[pos]:
                self.corrupt.append((self.turn, pos, ids[pos], got))
        self._step(params, blocks, computed, len(ids), session)
        for k in range(decode):
            cur = len(ids) + k
            if cur // BS >= len(blocks):
                blocks.append(self._block())
            self._put(blocks, cur, cur + 1, [1])
            self._step(params, blocks, cur, cur + 1, session)
        for k in range(len(ids) // BS):
            self.prefix.setdefault(tuple(ids[: (k + 1) * BS]), blocks[k])


def render(messages):
    return [t for m in messages for t in m] + [10]


def edit_plan(old, new):
    """One reused segment: the common suffix of ``old`` (minus its tail) moved into ``new``."""
    p = 0
    while p < min(len(old), len(new)) and old[p] == new[p]:
        p += 1
    s = 0
    while s < min(len(old), len(new)) - p and old[-1 - s] == new[-1 - s]:
        s += 1
    if s == 0:
        return None
    src, dst = len(old) - s, len(new) - s
    return {"dst_start": dst, "dst_end": dst + s, "delta": dst - src}


def run_session(turns: int, engine: Engine, session="s", front=True):
    msgs: list[list[int]] = []
    deltas = []
    counter = [1000]

    def message(n):
        counter[0] += 1
        return [counter[0] % 50000 + 11] * 3 + [(counter[0] * 7 + i) % 50000 + 11 for i in range(n)]

    for t in range(turns):
        engine.turn = t
        prev = render(msgs)
        if t >= 3:
            # demote the oldest full message (front shrink) or grow one in the middle
            k = 2 * (t - 3) % max(len(msgs), 1) if front else len(msgs) // 2
            msgs[k] = message(5 if front else len(msgs[k]) + 40)
            now = render(msgs)
            plan = edit_plan(prev, now)
            # the reused span is the unchanged tail of the history, before the new turn
            load = plan if plan and plan["dst_end"] - plan["dst_start"] >= BS else None
            if load:
                deltas.append(load["delta"])
            msgs.append(message(60))
            ids = render(msgs)
            if load:
                # the warm-up phase of an edit turn (reference server.py:407-411,
                # reuse_plan.phases): prefill the fresh span up to the block where the
                # segment begins, saving nothing, so vLLM's prefix hit lands there
                lo = -(-load["dst_start"] // BS) * BS
                hi = load["dst_end"] // BS * BS
                if hi - lo >= BS and 0 < lo and hi < len(ids):
                    engine.generate(ids[:lo], session, save=False, decode=1)
                    load = {"dst_start": lo, "dst_end": hi, "delta": load["delta"]}
                else:
                    load = None
            engine.generate(ids, session, load=load, save="full")
        else:
            msgs.append(message(60))
            engine.generate(render(msgs), session, save=True)
    return deltas


def test_thirty_front_edits_never_corrupt_a_position():
    e = Engine()
    deltas = run_session(30, e)
    assert e.corrupt == [], e.corrupt[:3]
    assert e.refused == 0
    assert e.loaded > 0, "no turn reused anything"
    assert min(deltas) < 0, "front demotions must move the tail earlier"


def test_mid_edits_grow_the_view_with_positive_deltas():
    e = Engine()
    deltas = run_session(20, e, front=False)
    assert e.corrupt == [] and e.refused == 0 and e.loaded > 0
    assert max(deltas) > 0


def test_sessions_coexist_without_thrashing():
    e = Engine(budget=24576)
    for t in range(3):
        for sid in ("a", "b", "c"):
            e.turn = t
            e.generate(render([[7 + t] * 300, [ord(sid)] * 200]), sid, save=True)
    assert e.store.evictions == 0 and e.corrupt == []
