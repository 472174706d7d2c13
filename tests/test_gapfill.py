"""Single-request multi-segment reuse: the gap plan the connector offers vLLM.

The connector's ``MARATHON_GAPFILL=1`` path hands every reused segment of a
request over at once; these are the plan's invariants, the ones the
reference's own gapfill tests pin (``tests/test_gapfill.py`` of the
reference): filled spans and computed positions partition the prompt
exactly, the engine always keeps the last position, spans too short to keep a
whole block are dropped rather than rounded outward, and the engine's own
prefix hit counts as filled.
"""

from __future__ import annotations

import pytest

from marathon_b200 import gapfill
from marathon_b200.gapfill import GapPlan, align, check, plan_gaps

BS = 16


def seg(lo: int, hi: int, delta: int = 0) -> dict:
    return {"dst_start": lo, "dst_end": hi, "delta": delta}


def _covered(plan: GapPlan) -> set[int]:
    return {i for lo, hi in plan.filled for i in range(lo, hi)}


def _partitions(plan: GapPlan, n: int) -> None:
    cov = _covered(plan)
    assert cov.isdisjoint(plan.compute)
    assert cov | set(plan.compute) == set(range(n))
    assert plan.compute[-1] == n - 1


def test_without_segments_everything_is_computed():
    p = plan_gaps([], BS, 300)
    assert p.filled == () and list(p.compute) == list(range(300)) and p.saving == 0.0


def test_one_segment_is_clipped_inward_to_blocks():
    p = plan_gaps([seg(100, 400)], BS, 1000)
    assert p.filled == ((112, 400),)  # 100 rounds up to 112; 400 is a boundary
    _partitions(p, 1000)
    assert p.filled_tokens + len(p.compute) == 1000


def test_several_segments_leave_exactly_their_complement():
    p = plan_gaps([seg(100, 400), seg(600, 900)], BS, 1000)
    assert p.filled == ((112, 400), (608, 896))
    _partitions(p, 1000)


def test_a_segment_shorter_than_a_block_after_clipping_is_dropped():
    p = plan_gaps([seg(100, 110)], BS, 400)
    assert p.filled == () and len(p.compute) == 400
    # 20 tokens that straddle a boundary keep no whole block either
    assert plan_gaps([seg(40, 60)], BS, 400).filled == ()


def test_the_final_block_always_stays_with_the_engine():
    p = plan_gaps([seg(0, 1000)], BS, 1000)
    assert p.filled[-1][1] <= (1000 - 1) // BS * BS
    assert p.compute[-1] == 999


def test_adjacent_and_overlapping_segments_merge():
    assert plan_gaps([seg(0, 256), seg(256, 512)], BS, 1000).filled == ((0, 512),)
    p = plan_gaps([seg(0, 300), seg(200, 512)], BS, 1000)
    assert p.filled == ((0, 512),) and p.filled_tokens == 512
    assert len(p.compute) == 1000 - 512


def test_segment_order_does_not_matter():
    assert plan_gaps([seg(600, 900), seg(100, 400)], BS, 1000) == \
        plan_gaps([seg(100, 400), seg(600, 900)], BS, 1000)


@pytest.mark.parametrize("n", [17, 64, 513, 1000, 7939])
@pytest.mark.parametrize("bs", [16, 32])
def test_partition_holds_for_any_prompt_and_block_size(n, bs):
    p = plan_gaps([seg(n // 8, n // 3), seg(n // 2, n - bs)], bs, n)
    _partitions(p, n)


def test_the_engines_own_prefix_hit_is_filled_not_recomputed():
    p = plan_gaps([seg(400, 800)], BS, 1000, local_hit=112)
    assert p.filled[0] == (0, 112) and min(p.compute) == 112
    _partitions(p, 1000)


def test_a_prefix_hit_merges_with_a_segment_starting_inside_it():
    p = plan_gaps([seg(64, 400)], BS, 1000, local_hit=128)
    assert p.filled == ((0, 400),) and p.compute[0] == 400


def test_a_prefix_hit_covering_the_prompt_still_leaves_the_last_token():
    p = plan_gaps([], BS, 500, local_hit=500)
    assert p.compute[-1] == 499 and p.filled_tokens + len(p.compute) == 500


def test_check_rejects_plans_a_scheduler_must_not_run():
    with pytest.raises(AssertionError):  # nothing left to compute
        check(GapPlan(filled=((0, 16),), compute=(), n_prompt=16))
    with pytest.raises(AssertionError):  # overlapping spans
        check(GapPlan(filled=((0, 16), (8, 32)), compute=(32,), n_prompt=33))
    with pytest.raises(AssertionError):  # duplicate / miscounted positions
        check(GapPlan(filled=((0, 16),), compute=(16, 16, 17), n_prompt=33))


def test_align_drops_negative_and_empty_spans():
    assert align([seg(-40, 10), seg(50, 50)], BS, 1000) == []
    assert align([seg(32, 96), seg(96, 160)], BS, 1000) == [(32, 160)]


def test_channel_hand_off_between_scheduler_and_worker():
    gapfill.clear()
    gapfill.offer("r1", [3, 4, 5], 96)
    pos, matched = gapfill.take("r1")
    assert list(pos) == [3, 4, 5] and matched == 96
    assert gapfill.take("r1") is None  # taken once
    gapfill.publish("r1", pos, matched)
    assert "r1" in gapfill.active() and gapfill.stats() == {"offered": 0, "active": 1}
    gapfill.offer("r2", [0], 0)
    gapfill.release("r1")
    gapfill.release("r2")
    assert gapfill.stats() == {"offered": 0, "active": 0}
