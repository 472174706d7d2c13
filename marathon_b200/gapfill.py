"""Non-prefix reuse for one request: which spans the connector fills, which vLLM computes.

Same contract as the reference's ``marathon.gapfill`` and
``marathon.gapfill_channel`` (``src/marathon/gapfill.py``,
``src/marathon/gapfill_channel.py``), which the connector's
``MARATHON_GAPFILL=1`` path consumes: a request's reused segments are clipped
inward to whole blocks, merged, and complemented into the exact list of
positions vLLM must still compute (always including the last prompt token).
The scheduler side of the reference's vLLM patch reads the plan through the
channel functions below; the loads themselves go through the same batched
kernel as any other load, all segments of the request in one launch.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

Span = tuple[int, int]


@dataclass(frozen=True)
class GapPlan:
    """Block-aligned ``filled`` spans and the ``compute`` positions, their exact complement."""

    filled: tuple[Span, ...]
    compute: tuple[int, ...]
    n_prompt: int

    @property
    def filled_tokens(self) -> int:
        return sum(hi - lo for lo, hi in self.filled)

    @property
    def saving(self) -> float:
        return self.filled_tokens / self.n_prompt if self.n_prompt else 0.0


def align(loads: list[dict], block_size: int, n_prompt: int) -> list[Span]:
    """Clip each load inward to block boundaries, never claiming the prompt's last block.

    Spans left with less than one block are dropped; the rest are sorted and
    overlapping or touching spans merged (``gapfill.py:57-79``).
    """
    last_claimable = (n_prompt - 1) // block_size * block_size
    spans = []
    for ld in loads:
        lo = -(-int(ld["dst_start"]) // block_size) * block_size
        hi = min(int(ld["dst_end"]), last_claimable) // block_size * block_size
        if lo >= 0 and hi - lo >= block_size:
            spans.append((lo, hi))
    spans.sort()
    merged: list[Span] = []
    for lo, hi in spans:
        if merged and lo <= merged[-1][1]:
            merged[-1] = (merged[-1][0], max(merged[-1][1], hi))
        else:
            merged.append((lo, hi))
    return merged


def plan_gaps(loads: list[dict], block_size: int, n_prompt: int, local_hit: int = 0) -> GapPlan:
    """Filled spans (vLLM's own prefix hit counts as filled) and the positions to compute."""
    filled = align(loads, block_size, n_prompt)
    if local_hit > 0:
        filled = align(
            [{"dst_start": 0, "dst_end": min(local_hit, n_prompt)}]
            + [{"dst_start": lo, "dst_end": hi} for lo, hi in filled],
            block_size,
            n_prompt,
        )
    compute: list[int] = []
    cursor = 0
    for lo, hi in filled:
        compute.extend(range(cursor, lo))
        cursor = hi
    compute.extend(range(cursor, n_prompt))
    plan = GapPlan(tuple(filled), tuple(compute), n_prompt)
    check(plan)
    return plan


def check(plan: GapPlan) -> None:
    """The invariants a patched scheduler relies on (``gapfill.py:109-122``)."""
    prev = 0
    for lo, hi in plan.filled:
        if not 0 <= lo < hi <= plan.n_prompt:
            raise AssertionError(f"bad span {(lo, hi)} in {plan.n_prompt}")
        if lo < prev:
            raise AssertionError(f"spans out of order or overlapping at {(lo, hi)}")
        prev = hi
    if not plan.compute or plan.compute[-1] != plan.n_prompt - 1:
        raise AssertionError("the engine must always be left the final position to compute")
    if len(plan.compute) + plan.filled_tokens != plan.n_prompt:
        raise AssertionError("computed + filled != prompt length")
    if len(set(plan.compute)) != len(plan.compute):
        raise AssertionError("duplicate compute positions")


# ------------------------------------------------------------------ channel
# request id -> (positions the engine must compute, tokens the connector fills);
# a module-level hand-off is valid because vLLM's v1 scheduler and worker share
# a process in the single-GPU configuration this path supports.
_offered: dict[str, tuple[np.ndarray, int]] = {}
_active: dict[str, tuple[np.ndarray, int]] = {}


def offer(request_id: str, positions, matched: int) -> None:
    _offered[str(request_id)] = (np.asarray(positions, dtype=np.int64), int(matched))


def take(request_id: str) -> tuple[np.ndarray, int] | None:
    return _offered.pop(str(request_id), None)


def publish(request_id: str, positions, matched: int) -> None:
    _active[str(request_id)] = (np.asarray(positions, dtype=np.int64), int(matched))


def active() -> dict[str, tuple[np.ndarray, int]]:
    return _active


def release(request_id: str) -> None:
    rid = str(request_id)
    _offered.pop(rid, None)
    _active.pop(rid, None)


def clear() -> None:
    _offered.clear()
    _active.clear()


def stats() -> dict[str, int]:
    return {"offered": len(_offered), "active": len(_active)}
