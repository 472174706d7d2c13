"""Session-keyed, position-indexed KV store with a token budget and whole-session LRU.

Drop-in for the reference's ``marathon.shift_store`` (``src/marathon/shift_store.py``):
same names, same arguments, same answers.  Bookkeeping (``reserve``,
``covers``, growth, eviction, counters) stays on the host exactly as specified
there; what changes is who moves the bytes.  The connector never builds a
gathered ``[n, heads, 2*head_size]`` tensor: the native save kernel writes
paged rows straight into the buffers below, and the native load kernel reads
them straight out, every layer of a step in one launch.  :meth:`ShiftStore.view`
is the bridge — it hands those kernels the buffers' device addresses.

Storage per session is one buffer per layer, ``[capacity, heads, 2*head_size]``,
row = absolute token position (``shift_store.py:12-17``).  ``write`` / ``read``
keep the reference's tensor-level contract for callers that already hold a
gathered tensor; they are plain tensor copies / views on whatever device the
store lives on.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np
import torch

# Capacity floor of a session's first allocation; capacities then double
# (shift_store.py:41-52 records why: fixed steps and big fixed slabs both
# thrash the allocator, geometric growth from a small floor does not).
SLAB = 2048
DEFAULT_STORE_TOKENS = 32768


def _settle_host_copies(buffers) -> None:
    """Before a host-tier buffer is copied on the CPU (growth), let the GPU finish
    the staged copies that may still be writing it."""
    if torch.cuda.is_available() and any(not b.is_cuda for b in buffers):
        torch.cuda.synchronize()


def slots(block_ids: list[int], lo: int, hi: int, block_size: int) -> torch.Tensor:
    """Flat slot indices of positions ``[lo, hi)`` through a block table (int64, host).

    ``table[p // bs] * bs + p % bs`` (``shift_store.py:56-60``).  The batched
    kernels compute the same numbers on the device from the block table.
    """
    pos = torch.arange(lo, hi, dtype=torch.int64)
    table = torch.as_tensor(block_ids, dtype=torch.int64)
    return table[pos // block_size] * block_size + (pos % block_size)


class SessionTable:
    """One in-flight writer per session, keyed by request id (``shift_store.py:63-90``)."""

    def __init__(self) -> None:
        self._owner: dict[str, str] = {}  # session -> request id holding it
        self._session: dict[str, str] = {}  # request id -> session it holds
        self.conflicts = 0

    def acquire(self, request_id: str, session: str) -> bool:
        """Claim ``session`` for ``request_id``; False if another request holds it."""
        holder = self._owner.get(session)
        if holder is not None and holder != request_id:
            self.conflicts += 1
            return False
        self._owner[session] = request_id
        self._session[request_id] = session
        return True

    def session_of(self, request_id: str) -> str | None:
        return self._session.get(request_id)

    def release(self, request_id: str) -> None:
        session = self._session.pop(request_id, None)
        if session is not None and self._owner.get(session) == request_id:
            del self._owner[session]

    def __len__(self) -> int:
        return len(self._owner)


@dataclass
class _Entry:
    capacity: int = 0  # positions each layer buffer can hold
    base: int = -1  # first position ever written (-1: nothing yet)
    filled: int = 0  # [base, filled) holds valid KV of the current history
    layers: dict[str, torch.Tensor] = field(default_factory=dict)


class ShiftStore:
    """Position-indexed KV per session under a total token budget, LRU across sessions.

    Constructor and semantics of ``shift_store.py:101-266``.  ``allocate=False``
    is the scheduler-side mirror: identical bookkeeping, no tensors.
    """

    def __init__(
        self,
        budget_tokens: int = DEFAULT_STORE_TOKENS,
        device: str = "cuda",
        allocate: bool = True,
        slab: int | None = None,
        session_cap: int | None = None,
    ) -> None:
        self.budget = int(budget_tokens)
        self.slab = min(int(slab or SLAB), self.budget)
        # a known per-session ceiling is allocated up front so later saves never
        # grow a buffer; it is a floor for growth, not a cap (shift_store.py:114-123)
        self.session_cap = min(int(session_cap), self.budget) if session_cap else 0
        self.device = device
        self.allocate = allocate
        self._sessions: OrderedDict[str, _Entry] = OrderedDict()  # oldest first
        # bumped whenever a buffer is created, replaced or dropped: the cached
        # pointer view handed to the native kernels is valid while it is unchanged
        self._version = 0
        self._view_cache: tuple | None = None
        self.hits = 0
        self.misses = 0
        self.evictions = 0
        self.refusals = 0
        self.loaded_token_layers = 0
        self.saved_token_layers = 0

    # ------------------------------------------------------------ internals
    def _touch(self, session: str) -> _Entry:
        entry = self._sessions.get(session)
        if entry is None:
            entry = self._sessions[session] = _Entry()
        else:
            self._sessions.move_to_end(session)
        return entry

    @property
    def used(self) -> int:
        return sum(e.capacity for e in self._sessions.values())

    def _grow(self, session: str, entry: _Entry, want: int) -> None:
        """Grow ``session`` to hold ``want`` positions (``shift_store.py:149-175``).

        New capacity: the largest of the session cap, the slab floor and twice
        the current capacity, doubled until it covers ``want``, then clipped to
        the budget.  Least-recently-used *other* sessions are evicted until it
        fits; stored rows ``[0, filled)`` survive the reallocation.
        """
        size = max(self.session_cap, self.slab, entry.capacity * 2)
        while size < want:
            size *= 2
        new_cap = min(self.budget, size)
        while self.used - entry.capacity + new_cap > self.budget:
            victim = next((s for s in self._sessions if s != session), None)
            if victim is None:
                break
            self.drop(victim)
            self.evictions += 1
        keep = entry.filled
        self._version += 1
        _settle_host_copies(entry.layers.values())
        for name, old in list(entry.layers.items()):
            fresh = self.new_buffer((new_cap, *old.shape[1:]), old.dtype, old.device)
            n = min(keep, old.shape[0])
            fresh[:n] = old[:n]
            entry.layers[name] = fresh
        entry.capacity = new_cap

    # --------------------------------------------------------------- public
    def reserve(self, session: str, dst_start: int, n: int) -> bool:
        """Make room for positions ``[dst_start, dst_start + n)`` (``shift_store.py:179-206``).

        Refused (False, nothing stored) when the span exceeds the budget on its
        own, is empty, or would leave a hole above ``filled``.  A span starting
        at or below ``filled`` truncates everything above it: that is an edit.
        Idempotent for a repeated ``(session, dst_start, n)``.
        """
        need = dst_start + n
        entry = self._touch(session)
        first = entry.base < 0
        if need > self.budget or n <= 0 or (not first and dst_start > entry.filled):
            self.refusals += 1
            return False
        if need > entry.capacity:
            self._grow(session, entry, need)
        if first:
            # the first save starts at the request's prefix-cache hit, never
            # below it: the store must not claim the head it never wrote
            entry.base = dst_start
        entry.filled = need
        return True

    def truncate(self, session: str, pos: int) -> None:
        """Forget ``session``'s positions from ``pos`` on: a save there did not land.

        The session keeps ``[base, min(filled, pos))``.  A later save that
        starts above that is refused by :meth:`reserve` (it would leave a
        hole), and a load reaching past it is declined by :meth:`covers`, so
        the lost span is recomputed, never loaded.  Idempotent; the scheduler
        mirror and the worker store apply the same truncations.  (The
        reference has no such path: its saves were synchronous torch copies.)
        """
        entry = self._sessions.get(session)
        if entry is None or entry.base < 0:
            return
        entry.filled = max(entry.base, min(entry.filled, int(pos)))

    def covers(self, session: str, start: int, n: int) -> bool:
        """Whether ``[start, start + n)`` is held for ``session`` (``shift_store.py:208-223``)."""
        entry = self._sessions.get(session)
        ok = (
            entry is not None
            and entry.base >= 0
            and start >= entry.base
            and n > 0
            and start + n <= entry.filled
        )
        if ok:
            self.hits += 1
            self._touch(session)
        else:
            self.misses += 1
        return ok

    def write(self, session: str, layer: str, dst_start: int, src: torch.Tensor) -> None:
        """Copy a gathered ``[n, heads, 2*head_size]`` tensor into the session's buffer."""
        entry = self._sessions.get(session)
        n = src.shape[0]
        if entry is None or dst_start + n > entry.capacity or not self.allocate:
            return
        buf = self._buffer(entry, layer, src.shape[1:], src.dtype)
        # a host-tier buffer is written synchronously: it may be regrown (a CPU
        # copy) before the stream would have finished a non-blocking write
        buf[dst_start : dst_start + n] = src.to(buf.device, non_blocking=buf.is_cuda)
        self.saved_token_layers += n

    def read(self, session: str, layer: str, start: int, n: int) -> torch.Tensor | None:
        """View of rows ``[start, start + n)`` or None if not held (``shift_store.py:238-250``)."""
        entry = self._readable(session, start, n)
        if entry is None:
            return None
        buf = entry.layers.get(layer)
        if buf is None:
            return None
        self.loaded_token_layers += n
        # same touch order as the scheduler mirror's covers(), so both LRU
        # orders -- and therefore both eviction choices -- stay identical
        self._touch(session)
        return buf[start : start + n]

    def drop(self, session: str) -> None:
        if self._sessions.pop(session, None) is not None:
            self._version += 1

    def stats(self) -> dict:
        return {
            "budget_tokens": self.budget,
            "used_tokens": self.used,
            "sessions": {s: max(e.filled - max(e.base, 0), 0) for s, e in self._sessions.items()},
            "hits": self.hits,
            "misses": self.misses,
            "evictions": self.evictions,
            "refusals": self.refusals,
            "loaded_token_layers": self.loaded_token_layers,
            "saved_token_layers": self.saved_token_layers,
        }

    # ------------------------------------------- native-kernel bridge
    def _readable(self, session: str, start: int, n: int) -> _Entry | None:
        entry = self._sessions.get(session)
        if entry is None or entry.base < 0 or start < entry.base or start + n > entry.filled:
            return None
        return entry

    def new_buffer(self, shape, dtype, device) -> torch.Tensor:
        """A zeroed buffer; on the host tier (``device="cpu"``) pinned when CUDA is up,
        so the staged copies to and from the GPU run on the copy engines."""
        if torch.device(device).type == "cpu" and torch.cuda.is_available():
            return torch.zeros(shape, dtype=dtype, pin_memory=True)
        return torch.zeros(shape, dtype=dtype, device=device)

    def _buffer(self, entry: _Entry, layer: str, row_shape, dtype) -> torch.Tensor:
        buf = entry.layers.get(layer)
        if buf is None:
            buf = self.new_buffer((entry.capacity, *row_shape), dtype, self.device)
            entry.layers[layer] = buf
            self._version += 1
        return buf

    def ensure_layers(
        self, session: str, layers: list[str], heads: int, row: int, dtype: torch.dtype
    ) -> bool:
        """Allocate any missing layer buffer of ``session`` (what ``write`` does lazily)."""
        entry = self._sessions.get(session)
        if entry is None or not self.allocate or entry.capacity <= 0:
            return False
        for name in layers:
            self._buffer(entry, name, (heads, row), dtype)
        return True

    def loadable(self, session: str, layers: list[str], start: int, n: int,
                 layer_set: frozenset | None = None) -> str | None:
        """First layer whose rows ``[start, start + n)`` cannot be read, or None.

        The batched load checks a whole load before launching, where the
        reference's per-layer ``read`` discovered a gap mid-loop.  ``layer_set``
        is ``layers`` as a set, for callers that check many loads.
        """
        entry = self._readable(session, start, n)
        if entry is not None and entry.layers.keys() >= (layer_set or set(layers)):
            return None
        for name in layers:
            if entry is None or name not in entry.layers:
                return name
        return None

    def mark_loaded(self, session: str, layers: list[str], n: int) -> None:
        """Counters and LRU position after one ``read`` per layer (``shift_store.py:245-249``).

        Touching the same session once or once per layer leaves the same LRU
        order, so it is touched once.
        """
        self.loaded_token_layers += n * len(layers)
        if layers:
            self._touch(session)

    def adopt(self, session: str, layers: dict[str, torch.Tensor], base: int, filled: int) -> None:
        """Register already-filled buffers for ``session`` as holding ``[base, filled)``.

        For harnesses that build a session's rows elsewhere (benchmarks,
        tests); the buffers count against the budget like any other.
        """
        caps = {t.shape[0] for t in layers.values()}
        if len(caps) != 1:
            raise ValueError("adopted layer buffers must share one capacity")
        entry = self._touch(session)
        entry.capacity = caps.pop()
        entry.base, entry.filled = int(base), int(filled)
        entry.layers = dict(layers)
        self._version += 1

    def mark_saved(self, n_tokens: int, n_layers: int) -> None:
        self.saved_token_layers += n_tokens * n_layers

    def capacity(self, session: str) -> int:
        entry = self._sessions.get(session)
        return entry.capacity if entry is not None else 0

    def view(self, sessions: list[str], layers: list[str]):
        """Device addresses of ``sessions`` x ``layers`` buffers for the native kernels.

        Missing buffers are address 0, which the kernels reject per tile
        (``MSHIFT_EBIT_SESSION``) instead of dereferencing.
        """
        from .shift_kernels import StoreView

        key = (tuple(sessions), tuple(layers))
        cached = self._view_cache
        if cached is not None and cached[0] == key and cached[1] == self._version:
            return cached[2]
        ptrs = np.zeros((len(sessions), len(layers)), dtype=np.uint64)
        caps = np.zeros(len(sessions), dtype=np.int64)
        st_tok = st_head = None
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
                if st_tok is None:
                    st_tok, st_head = buf.stride(0), buf.stride(1)
                elif (st_tok, st_head) != (buf.stride(0), buf.stride(1)):
                    raise ValueError("store buffers of one batch must share a row layout")
        view = StoreView(ptrs, caps, st_tok or 0, st_head or 0, keep)
        self._view_cache = (key, self._version, view)
        return view


@dataclass(frozen=True)
class LoadDecision:
    """A resolved load: destination ``[lo, hi)``, source at ``lo - delta``."""

    lo: int
    hi: int
    delta: int

    @property
    def src_start(self) -> int:
        return self.lo - self.delta


def plan_load(
    store: ShiftStore,
    session: str | None,
    request: dict | None,
    num_computed: int,
    num_prompt_tokens: int,
    block_size: int,
) -> tuple[LoadDecision | None, str]:
    """Decide whether a request's ``load`` can be served (``shift_store.py:282-315``).

    ``None`` always means recompute, never guess.  The served span starts at
    vLLM's own prefix hit ``num_computed`` and ends at the last whole block
    that still leaves one prompt token for vLLM to compute.
    """
    if not session or not request:
        return None, "no session or no load requested"
    lo = int(num_computed)
    dst_end = int(request["dst_end"])
    delta = int(request["delta"])
    if num_computed < int(request["dst_start"]):
        return None, f"local hit {num_computed} < dst_start {request['dst_start']}"
    hi = min(dst_end, (num_prompt_tokens - 1) // block_size * block_size)
    hi -= hi % block_size
    if hi <= lo:
        return None, f"nothing left after block alignment (hi={hi} <= lo={lo})"
    if not store.covers(session, lo - delta, hi - lo):
        return None, f"store no longer holds [{lo - delta},{hi - delta})"
    return LoadDecision(lo, hi, delta), "ok"


def plan_save(
    store: ShiftStore, session: str | None, mode: object, lo: int, hi: int
) -> tuple[int, int] | None:
    """Position range a step saves (``shift_store.py:318-333``); ``"full"`` widens to 0."""
    if hi <= lo or not session or not mode:
        return None
    if mode == "full":
        lo = 0
    if not store.reserve(session, lo, hi - lo):
        return None
    return lo, hi


def churn_tokens(loads: list[dict]) -> tuple[int, int]:
    """``(changed_before_span, span_len)`` of one turn's loads (``shift_store.py:336-357``).

    ``span_len`` is the total reused length; ``changed_before_span`` the
    positions before the deepest reused segment that this plan does not reuse.
    """
    if not loads:
        return 0, 0
    spans = sorted((int(d["dst_start"]), int(d["dst_end"])) for d in loads)
    span_len = sum(hi - lo for lo, hi in spans)
    deepest = spans[-1][0]
    reused_before = sum(min(hi, deepest) - lo for lo, hi in spans if lo < deepest)
    return max(0, deepest - reused_before), span_len
