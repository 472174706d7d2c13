"""Single-request multi-segment reuse: the gap plan handed to a patched vLLM.

With ``gapfill`` on, a request's ``"loads"`` are served in one request: the
connector plans the filled spans and the positions vLLM must still compute
with the reference's ``marathon.gapfill.plan_gaps`` and offers that plan on
``marathon.gapfill_channel``, the module the reference's vLLM patch reads
(``scripts/patch_vllm_gapfill.py:60-68`` in the scheduler, ``:82-84`` in the
model runner).  These tests play that patched scheduler and runner against the
reference's own channel module, then run the worker's load on the GPU, and
check the decline paths: no channel, or a vLLM without the patch, means 0
matched tokens, never a non-prefix span passed off as a prefix.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

vllm_base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")
KVConnectorRole = vllm_base.KVConnectorRole

from marathon_b200 import vllm_shift_connector as C  # noqa: E402
from parity import reference_tables  # noqa: E402
from vllm_fakes import BS, fake_config, forward_context, new_req, request, sched_output  # noqa: E402

N_PROMPT = 2000
LOADS = [{"dst_start": 100, "dst_end": 600, "delta": 20},
         {"dst_start": 700, "dst_end": 1500, "delta": -40},
         {"dst_start": 1600, "dst_end": 1605, "delta": 3}]  # under a block: dropped


def _scheduler(**extra):
    cfg = {"store_tokens": 65536, "gapfill": True, **extra}
    return C.MarathonShiftConnector(fake_config(cfg), KVConnectorRole.SCHEDULER, None)


def _offer(conn, rid="g", computed=0, loads=LOADS):
    conn._store.reserve("s", 0, N_PROMPT)  # the history a previous turn saved
    r = request(rid, {"session": "s", "loads": loads}, N_PROMPT)
    conn.on_new_request(r)
    return r, conn.get_num_new_matched_tokens(r, computed)


def test_declines_when_the_channel_module_is_missing():
    conn = _scheduler(gapfill_channel="marathon_no_such.gapfill_channel",
                      gapfill_require_patch=False)
    _, got = _offer(conn)
    assert got == (0, False)
    assert conn._multi == {}
    assert "gap-fill channel unavailable" in conn._gap.why


def test_declines_when_vllm_lacks_the_patch(reference_pkg):
    channel = importlib.import_module("marathon.gapfill_channel")
    channel.clear()
    assert not C.GapHandoff.vllm_patched()  # the vLLM installed here is unpatched
    conn = _scheduler()
    _, got = _offer(conn)
    assert got == (0, False)
    assert channel.stats() == {"offered": 0, "active": 0}
    assert "patch" in conn._gap.why


def test_single_segment_loads_are_unaffected_by_a_missing_channel():
    conn = _scheduler(gapfill_channel="marathon_no_such.gapfill_channel")
    conn._store.reserve("s", 0, N_PROMPT)
    r = request("one", {"session": "s", "load": {"dst_start": 64, "dst_end": 1024,
                                                 "delta": 32}}, N_PROMPT)
    conn.on_new_request(r)
    assert conn.get_num_new_matched_tokens(r, 64) == (1024 - 64, False)


def _play_patched_vllm(channel, rid):
    """What the patched scheduler and model runner do with an offer."""
    taken = channel.take(rid)  # scheduler: consume the offer ...
    assert taken is not None
    positions, matched = taken
    channel.publish(rid, positions, matched)  # ... and publish it for the runner
    assert channel.take(rid) is None  # an offer is taken once
    return channel.active()[rid]  # runner: the positions to compute


def test_plan_reaches_the_patched_scheduler_and_runner(reference_pkg):
    channel = importlib.import_module("marathon.gapfill_channel")
    channel.clear()
    conn = _scheduler(gapfill_require_patch=False)  # stands in for a patched vLLM
    r, (n, async_) = _offer(conn)
    assert async_ is False
    accepted = conn._multi["g"]
    assert [(a["dst_start"], a["dst_end"]) for a in accepted] == [(112, 592), (704, 1488)]
    assert n == (592 - 112) + (1488 - 704)
    positions, matched = _play_patched_vllm(channel, "g")
    assert matched == n
    conn.update_state_after_alloc(r, None, n)
    meta = conn.build_connector_meta(sched_output([new_req("g", range(200), matched)],
                                                  scheduled={"g": N_PROMPT - n}))
    assert [(ld.src_start, ld.delta, ld.dst_start, ld.length) for ld in meta.loads] == [
        (92, 20, 112, 480), (744, -40, 704, 784)]
    filled = {p for ld in meta.loads for p in range(ld.dst_start, ld.dst_start + ld.length)}
    computed = set(int(p) for p in positions)
    assert len(computed) == len(positions) == N_PROMPT - n
    assert filled.isdisjoint(computed) and filled | computed == set(range(N_PROMPT))
    assert int(positions[-1]) == N_PROMPT - 1  # vLLM always computes the last token
    conn.request_finished(r, [])
    assert channel.stats() == {"offered": 0, "active": 0}


def test_prefix_hit_counts_as_filled(reference_pkg):
    channel = importlib.import_module("marathon.gapfill_channel")
    channel.clear()
    conn = _scheduler(gapfill_require_patch=False)
    _, (n, _) = _offer(conn, computed=128)
    positions, matched = _play_patched_vllm(channel, "g")
    # the engine's own 128-token prefix is filled, not recomputed
    assert min(int(p) for p in positions) >= 128 and 0 not in set(positions.tolist())
    assert matched - 128 == n
    channel.release("g")


@pytest.mark.gpu
def test_gap_filled_request_loads_every_segment_bit_exact(cuda, reference_pkg):
    """Scheduler plan -> patched-vLLM hand-off -> one worker load on the GPU.

    The loaded spans and the positions vLLM computes partition the prompt;
    every loaded position holds the oracle's rotation of its store row, and
    every position left to compute is untouched.
    """
    from oracle import shift_oracle as O

    channel = importlib.import_module("marathon.gapfill_channel")
    channel.clear()
    sched = _scheduler(gapfill_require_patch=False)
    r, (n, _) = _offer(sched)
    positions, matched = _play_patched_vllm(channel, "g")
    sched.update_state_after_alloc(r, None, n)
    H, D, L, NBLK = 8, 128, 3, 160
    blocks = np.random.default_rng(5).permutation(NBLK)[:N_PROMPT // BS + 1].tolist()
    meta = sched.build_connector_meta(sched_output([new_req("g", blocks, matched)],
                                                   scheduled={"g": N_PROMPT - n}))

    worker = C.MarathonShiftConnector(fake_config({"store_tokens": 65536, "gapfill": True}),
                                      KVConnectorRole.WORKER, None)
    g = torch.Generator().manual_seed(11)
    caches = {f"model.layers.{i}.self_attn.attn":
              torch.randn(NBLK, BS, H, 2 * D, generator=g).to(torch.bfloat16).to(cuda)
              for i in range(L)}
    worker.register_kv_caches(caches)
    store = worker._store
    assert store.reserve("s", 0, N_PROMPT)
    assert store.ensure_layers("s", list(caches), H, 2 * D, torch.bfloat16)
    rows = {}
    for name in caches:
        buf = store._sessions["s"].layers[name]
        buf.copy_(torch.randn(buf.shape, generator=g).to(torch.bfloat16))
        rows[name] = buf[:N_PROMPT].cpu().view(torch.int16).numpy().view(np.uint16)
    snap = {name: kv.cpu().view(torch.int16).numpy().view(np.uint16) for name, kv in caches.items()}

    worker.bind_connector_metadata(meta)
    worker.start_load_kv(forward_context())
    worker.wait_for_save()
    worker.clear_connector_metadata()
    torch.cuda.synchronize()
    assert worker.get_block_ids_with_load_errors() == set()

    inv = worker._inv_freq.numpy()
    bt = np.asarray(blocks)
    filled = np.zeros(N_PROMPT, dtype=bool)
    for name, kv in caches.items():
        got = kv.cpu().view(torch.int16).numpy().view(np.uint16)
        for ld in meta.loads:
            pos = np.arange(ld.dst_start, ld.dst_start + ld.length)
            filled[pos] = True
            src = rows[name][ld.src_start : ld.src_start + ld.length]
            tab = reference_tables([ld.delta], inv, cuda)[0]
            at = got[bt[pos // BS], pos % BS]
            assert np.array_equal(at[..., D:], src[..., D:]), name
            assert np.array_equal(at[..., :D], O.shift_k_bits(src[..., :D], tab, O.BF16)), name
        rest = np.asarray(positions)
        assert np.array_equal(got[bt[rest // BS], rest % BS], snap[name][bt[rest // BS], rest % BS])
    assert not filled[np.asarray(positions)].any()
    assert filled.sum() + len(positions) == N_PROMPT
    channel.release("g")
