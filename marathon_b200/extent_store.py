"""Generation-tagged interval store: reuse from generation-0 keys without re-saving.

The reference's ``ShiftStore`` is a flat ``[base, filled)`` window per session
whose row ``i`` holds the keys computed at position ``i``
(``src/marathon/shift_store.py:101-266``).  A save at a lower position
truncates everything above it, so a turn that reuses spans must re-save them
(``"full"``) and the store fills with rotated copies of rotated copies; the
reference's ``remap`` module (``src/marathon/remap.py``) would avoid that, but
it cannot be wired to a flat window, and its server refuses
``resave=False`` (``src/marathon/server.py:262-276``;
``docs/single-request-load.md``, "What unblocking costs").

This module is the missing store.  Keys are kept as **extents**: rows of a
session buffer allocated from a free list, each tagged with the generation
(turn) that computed them and the position they were computed at (``pos0``).
A fresh span saved in generation ``g`` never overwrites another generation's
rows, and a reused span is loaded from the rows of the generation that
computed it, rotated once by ``delta = new position - pos0``.  So reuse can go
on for any number of turns and every load re-rotates generation-0 bytes.

* :class:`ExtentStore` -- the store: per-session buffers (``[capacity,
  heads, 2*head_size]`` per layer, as ``ShiftStore``) with extents, a free
  list, geometric growth, a token budget and LRU eviction across sessions.
  ``allocate=False`` is the scheduler-side mirror; both sides run the same
  ``save_extent`` / ``release`` calls in the same order and so allocate the
  same rows.
* :class:`AddressBook` -- the server-side map from a session's logical
  positions to ``(generation, pos0)``; it turns a turn's reused segments into
  loads tagged with their generation and reports which extents fell out of
  the view (to ``release``).

The kernels and the worker are unchanged: a load is a run with its own store
row and delta, which they already take separately.
"""

from __future__ import annotations

import bisect
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np
import torch

from .shift_store import SLAB, _settle_host_copies


@dataclass
class _Ext:
    gen: int
    pos0: int  # first position the rows were computed at
    n: int
    row: int  # first store row

    @property
    def end(self) -> int:
        return self.pos0 + self.n


@dataclass
class _Session:
    capacity: int = 0
    layers: dict = field(default_factory=dict)
    # gen -> extents sorted by pos0, non-overlapping in pos0
    extents: dict = field(default_factory=dict)
    # free row intervals [lo, hi), sorted, disjoint, never adjacent
    free: list = field(default_factory=list)

    def used_rows(self) -> int:
        return sum(e.n for exts in self.extents.values() for e in exts)


class ExtentStore:
    """Per-session KV rows allocated as generation-tagged extents under a token budget."""

    def __init__(self, budget_tokens: int, device: str = "cuda", allocate: bool = True,
                 slab: int | None = None) -> None:
        self.budget = int(budget_tokens)
        self.slab = min(int(slab or SLAB), self.budget)
        self.device = device
        self.allocate = allocate
        self._sessions: OrderedDict[str, _Session] = OrderedDict()
        self._version = 0
        self._view_cache: tuple | None = None
        self.hits = self.misses = self.evictions = self.refusals = 0
        self.loaded_token_layers = self.saved_token_layers = 0

    # ------------------------------------------------------------ internals
    @property
    def used(self) -> int:
        return sum(s.capacity for s in self._sessions.values())

    def _touch(self, session: str) -> _Session:
        entry = self._sessions.get(session)
        if entry is None:
            entry = self._sessions[session] = _Session()
        else:
            self._sessions.move_to_end(session)
        return entry

    def new_buffer(self, shape, dtype, device) -> torch.Tensor:
        if torch.device(device).type == "cpu" and torch.cuda.is_available():
            return torch.zeros(shape, dtype=dtype, pin_memory=True)
        return torch.zeros(shape, dtype=dtype, device=device)

    def _free_rows(self, entry: _Session, lo: int, hi: int) -> None:
        """Return rows ``[lo, hi)`` to the free list, joining neighbours."""
        if hi <= lo:
            return
        free = entry.free
        i = bisect.bisect_left(free, (lo, hi))
        if i > 0 and free[i - 1][1] == lo:
            i -= 1
            lo = free[i][0]
            free.pop(i)
        if i < len(free) and free[i][0] == hi:
            hi = free[i][1]
            free.pop(i)
        free.insert(i, (lo, hi))

    def _take_rows(self, session: str, entry: _Session, n: int, after: int | None) -> int | None:
        """Allocate ``n`` contiguous rows: right after row ``after`` when free (an
        extent that keeps growing stays one run), else first fit, else grow."""
        if after is not None:
            for i, (lo, hi) in enumerate(entry.free):
                if lo == after and hi - lo >= n:
                    entry.free[i] = (lo + n, hi)
                    if lo + n == hi:
                        entry.free.pop(i)
                    return lo
        for i, (lo, hi) in enumerate(entry.free):
            if hi - lo >= n:
                entry.free[i] = (lo + n, hi)
                if lo + n == hi:
                    entry.free.pop(i)
                return lo
        if not self._grow(session, entry, n):
            return None
        return self._take_rows(session, entry, n, after)

    def _grow(self, session: str, entry: _Session, n: int) -> bool:
        """Enlarge the session so ``n`` more contiguous rows fit at its end.

        The new capacity doubles (from the slab floor) until the tail free run
        holds ``n``; other sessions are evicted least-recently-used first while
        the budget is exceeded.  Rows keep their indices.
        """
        tail = entry.free[-1][1] - entry.free[-1][0] if entry.free and \
            entry.free[-1][1] == entry.capacity else 0
        need = entry.capacity - tail + n
        size = max(self.slab, entry.capacity * 2)
        while size < need:
            size *= 2
        size = min(size, self.budget)
        if size < need:
            self.refusals += 1
            return False
        while self.used - entry.capacity + size > self.budget:
            victim = next((s for s in self._sessions if s != session), None)
            if victim is None:
                self.refusals += 1
                return False
            self.drop(victim)
            self.evictions += 1
        old = entry.capacity
        self._version += 1
        _settle_host_copies(entry.layers.values())
        for name, buf in list(entry.layers.items()):
            fresh = self.new_buffer((size, *buf.shape[1:]), buf.dtype, buf.device)
            fresh[:old] = buf[:old]
            entry.layers[name] = fresh
        entry.capacity = size
        self._free_rows(entry, old, size)
        return True

    # --------------------------------------------------------------- public
    def save_extent(self, session: str, gen: int, pos0: int, n: int) -> list[tuple[int, int, int]]:
        """Rows for the keys generation ``gen`` computes at positions ``[pos0, pos0+n)``.

        Returns ``[(pos0, rows, first_row), ...]`` covering the span, in
        position order: parts this generation already holds keep their rows
        (a repeated save is idempotent), new parts get new rows (extending the
        extent that ends at ``pos0`` in place when its next rows are free).
        Empty if the span cannot be held (budget); nothing is allocated then.
        """
        if n <= 0 or n > self.budget:
            self.refusals += 1 if n > 0 else 0
            return []
        entry = self._touch(session)
        exts = entry.extents.setdefault(gen, [])
        out: list[tuple[int, int, int]] = []
        cursor, end = pos0, pos0 + n
        i = bisect.bisect_right([e.pos0 for e in exts], pos0) - 1
        i = max(i, 0)
        while cursor < end:
            # an existing extent of this generation covering `cursor`
            held = next((e for e in exts[i:] if e.pos0 <= cursor < e.end), None)
            if held is not None:
                take = min(end, held.end) - cursor
                out.append((cursor, take, held.row + cursor - held.pos0))
                cursor += take
                continue
            nxt = next((e.pos0 for e in exts if e.pos0 > cursor), end)
            take = min(end, nxt) - cursor
            prev = next((e for e in exts if e.end == cursor), None)
            row = self._take_rows(session, entry, take, prev.row + prev.n if prev else None)
            if row is None:
                return []
            if prev is not None and row == prev.row + prev.n:
                prev.n += take
            else:
                bisect.insort(exts, _Ext(gen, cursor, take, row), key=lambda e: e.pos0)
            out.append((cursor, take, row))
            cursor += take
        return out

    def locate(self, session: str, gen: int, pos0: int, n: int,
               count: bool = True) -> list[tuple[int, int, int]] | None:
        """Rows holding generation ``gen``'s keys of positions ``[pos0, pos0+n)``.

        ``[(pos0, rows, first_row), ...]`` in position order, or None (a miss)
        when any position is not held.
        """
        entry = self._sessions.get(session)
        exts = entry.extents.get(gen) if entry is not None else None
        out: list[tuple[int, int, int]] = []
        cursor, end = pos0, pos0 + n
        if exts and n > 0:
            for e in exts:
                if e.end <= cursor:
                    continue
                if e.pos0 > cursor:
                    break
                take = min(end, e.end) - cursor
                out.append((cursor, take, e.row + cursor - e.pos0))
                cursor += take
                if cursor >= end:
                    break
        ok = n > 0 and cursor >= end
        if count:
            if ok:
                self.hits += 1
                self._touch(session)
            else:
                self.misses += 1
        return out if ok else None

    def release(self, session: str, gen: int, pos0: int, n: int) -> int:
        """Free generation ``gen``'s rows of positions ``[pos0, pos0+n)``; returns rows freed."""
        entry = self._sessions.get(session)
        if entry is None or gen not in entry.extents or n <= 0:
            return 0
        lo, hi = pos0, pos0 + n
        kept: list[_Ext] = []
        freed = 0
        for e in entry.extents[gen]:
            a, b = max(e.pos0, lo), min(e.end, hi)
            if a >= b:
                kept.append(e)
                continue
            self._free_rows(entry, e.row + a - e.pos0, e.row + b - e.pos0)
            freed += b - a
            if e.pos0 < a:
                kept.append(_Ext(gen, e.pos0, a - e.pos0, e.row))
            if b < e.end:
                kept.append(_Ext(gen, b, e.end - b, e.row + b - e.pos0))
        if kept:
            entry.extents[gen] = kept
        else:
            del entry.extents[gen]
        return freed

    def drop(self, session: str) -> None:
        if self._sessions.pop(session, None) is not None:
            self._version += 1

    def stats(self) -> dict:
        return {
            "budget_tokens": self.budget,
            "used_tokens": self.used,
            "sessions": {s: e.used_rows() for s, e in self._sessions.items()},
            "generations": {s: sorted(e.extents) for s, e in self._sessions.items()},
            "hits": self.hits,
            "misses": self.misses,
            "evictions": self.evictions,
            "refusals": self.refusals,
            "loaded_token_layers": self.loaded_token_layers,
            "saved_token_layers": self.saved_token_layers,
        }

    # ------------------------------------------- the worker's store interface
    def capacity(self, session: str) -> int:
        entry = self._sessions.get(session)
        return entry.capacity if entry is not None else 0

    def ensure_layers(self, session: str, layers: list[str], heads: int, row: int,
                      dtype: torch.dtype) -> bool:
        entry = self._sessions.get(session)
        if entry is None or not self.allocate or entry.capacity <= 0:
            return False
        for name in layers:
            if name not in entry.layers:
                entry.layers[name] = self.new_buffer((entry.capacity, heads, row), dtype,
                                                     self.device)
                self._version += 1
        return True

    def loadable(self, session: str, layers: list[str], start: int, n: int,
                 layer_set: frozenset | None = None) -> str | None:
        """First layer lacking rows ``[start, start + n)`` of ``session``, or None.

        ``start`` is a store row here (the worker's load jobs carry rows that
        :meth:`locate` returned); the rows must lie inside allocated extents.
        """
        entry = self._sessions.get(session)
        ok = entry is not None and 0 <= start and start + n <= entry.capacity and n > 0
        if ok:
            for lo, hi in entry.free:
                if lo < start + n and start < hi:
                    ok = False
                    break
        if ok and entry.layers.keys() >= (layer_set or set(layers)):
            return None
        for name in layers:
            if not ok or name not in entry.layers:
                return name
        return None

    def mark_loaded(self, session: str, layers: list[str], n: int) -> None:
        self.loaded_token_layers += n * len(layers)
        if layers:
            self._touch(session)

    def mark_saved(self, n_tokens: int, n_layers: int) -> None:
        self.saved_token_layers += n_tokens * n_layers

    def view(self, sessions: list[str], layers: list[str]):
        """Device (or host-tier) addresses of ``sessions`` x ``layers`` buffers."""
        from .shift_kernels import StoreView

        key = (tuple(sessions), tuple(layers))
        cached = self._view_cache
        if cached is not None and cached[0] == key and cached[1] == self._version:
            return cached[2]
        ptrs = np.zeros((len(sessions), len(layers)), dtype=np.uint64)
        caps = np.zeros(len(sessions), dtype=np.int64)
        st = None
        keep = []
        for i, s in enumerate(sessions):
            entry = self._sessions.get(s)
            if entry is None:
                continue
            caps[i] = entry.capacity
            for j, name in enumerate(layers):
                buf = entry.layers.get(name)
                if buf is None:
                    continue
                ptrs[i, j] = buf.data_ptr()
                keep.append(buf)
                if st is None:
                    st = (buf.stride(0), buf.stride(1))
        view = StoreView(ptrs, caps, st[0] if st else 0, st[1] if st else 0, keep)
        self._view_cache = (key, self._version, view)
        return view


# ---------------------------------------------------------------- address book
#: ``(lo, hi, gen, pos0)``: logical ``[lo, hi)`` holds generation ``gen``'s keys
#: computed at positions ``[pos0, pos0 + hi - lo)``
Span = tuple[int, int, int, int]


@dataclass
class AddressBook:
    """A session's view: where each logical position's keys live, by generation.

    The server-side counterpart of :class:`ExtentStore` (what the reference's
    ``Remap`` is for offsets, ``src/marathon/remap.py:33-98``, with the
    generation made explicit so that fresh keys never need the rows of older
    ones).  Per turn: ``loads(segments)`` for the request's ``kv_transfer_params``,
    then ``after_turn(segments, total, gen)`` for the next turn, whose return
    value lists the extents that fell out of the view (to ``release``).
    """

    spans: list[Span] = field(default_factory=list)

    def translate(self, lo: int, hi: int) -> list[Span]:
        """The spans backing logical ``[lo, hi)`` in order; gaps are not held (gen -1)."""
        out: list[Span] = []
        cursor = lo
        for s_lo, s_hi, gen, pos0 in self.spans:
            if s_hi <= cursor or s_lo >= hi:
                continue
            if s_lo > cursor:
                out.append((cursor, min(s_lo, hi), -1, -1))
                cursor = min(s_lo, hi)
            end = min(s_hi, hi)
            if end > cursor:
                out.append((cursor, end, gen, pos0 + cursor - s_lo))
                cursor = end
            if cursor >= hi:
                break
        if cursor < hi:
            out.append((cursor, hi, -1, -1))
        return out

    def loads(self, segments: list[dict]) -> list[dict]:
        """Reused segments ``{dst_start, dst_end, delta}`` (positions before the turn
        at ``dst - delta``) as generation-tagged loads rotated from their ``pos0``."""
        out: list[dict] = []
        for seg in segments:
            lo, hi, delta = int(seg["dst_start"]), int(seg["dst_end"]), int(seg["delta"])
            for a, b, gen, pos0 in self.translate(lo - delta, hi - delta):
                if gen < 0:
                    continue  # never saved: recomputed, not loaded
                out.append({"dst_start": a + delta, "dst_end": b + delta,
                            "delta": a + delta - pos0, "gen": gen, "src_start": pos0})
        return out

    def after_turn(self, segments: list[dict], total: int,
                   gen: int) -> list[tuple[int, int, int]]:
        """Advance to the turn's new view; returns ``(gen, pos0, n)`` extents no
        longer referenced by it (for :meth:`ExtentStore.release`).

        Reused segments keep their generation and ``pos0`` at their new
        positions; every other position of ``[0, total)`` was computed (and
        saved) in generation ``gen`` at its own position.
        """
        moved: list[Span] = []
        for seg in segments:
            lo, hi, delta = int(seg["dst_start"]), int(seg["dst_end"]), int(seg["delta"])
            for a, b, g, pos0 in self.translate(lo - delta, hi - delta):
                if g >= 0:
                    moved.append((a + delta, b + delta, g, pos0))
        spans: list[Span] = []
        cursor = 0
        for a0, b, g, pos0 in sorted(moved):
            a, b = max(a0, cursor), min(b, total)
            if b <= a:
                continue
            if a > cursor:
                spans.append((cursor, a, gen, cursor))
            spans.append((a, b, g, pos0 + a - a0))
            cursor = b
        if cursor < total:
            spans.append((cursor, total, gen, cursor))
        # per generation, the pos0 intervals the new view references
        live: dict[int, list[tuple[int, int]]] = {}
        for a, b, g, p0 in spans:
            live.setdefault(g, []).append((p0, p0 + b - a))
        dead: list[tuple[int, int, int]] = []
        for a, b, g, p0 in self.spans:
            for lo, hi in _subtract((p0, p0 + b - a), sorted(live.get(g, []))):
                dead.append((g, lo, hi - lo))
        self.spans = _join(spans)
        return dead


def _subtract(iv: tuple[int, int], cuts: list[tuple[int, int]]) -> list[tuple[int, int]]:
    """``iv`` minus the (sorted) intervals ``cuts``."""
    out = []
    lo, hi = iv
    for c_lo, c_hi in cuts:
        if c_hi <= lo or c_lo >= hi:
            continue
        if c_lo > lo:
            out.append((lo, c_lo))
        lo = max(lo, c_hi)
        if lo >= hi:
            break
    if lo < hi:
        out.append((lo, hi))
    return out


def _join(spans: list[Span]) -> list[Span]:
    out: list[Span] = []
    for a, b, g, p in spans:
        if out and out[-1][1] == a and out[-1][2] == g and out[-1][3] + (a - out[-1][0]) == p:
            out[-1] = (out[-1][0], b, g, out[-1][3])
        else:
            out.append((a, b, g, p))
    return out
