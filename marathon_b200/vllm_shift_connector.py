"""vLLM KV connector for position-shifted KV reuse, running the sm_100a kernels.

Drop-in for the reference's ``marathon.vllm_shift_connector``: same class name,
same ``kv_transfer_params`` schema, same scheduler-side decisions, same store
bookkeeping and counters.  Register it with::

    KVTransferConfig(kv_connector="MarathonShiftConnector",
                     kv_connector_module_path="marathon_b200.vllm_shift_connector",
                     kv_role="kv_both",
                     kv_connector_extra_config={"store_tokens": ..., "session_tokens": ...})

Per request (``src/marathon/vllm_shift_connector.py:16-42``)::

    {"session": "<id>", "load": {"dst_start", "dst_end", "delta"},
     "loads": [...], "save": true | "full"}

What changes is the worker side:

* ``start_load_kv`` runs every load of the step x every layer in ONE native
  launch (``ShiftWorker.load``).  The reference launched one Triton kernel per
  layer per load after a per-layer ``ShiftStore.read`` and a per-load slot
  transfer (``:495-518``).  Here the request's block table (4 bytes per 16
  tokens) travels instead of a per-token slot tensor (8 bytes per token), in
  the batch's single descriptor copy; slots are formed on the device.
* ``save_kv_layer`` gathers the step's tokens for one layer straight from the
  paged cache into the store buffer (one launch, no intermediate tensor).
  With ``kv_connector_extra_config["batch_save"]`` (or
  ``MARATHON_BATCH_SAVE=1``) the per-layer saves are deferred to
  ``wait_for_save`` and run as one launch over all layers.
* ``store_device`` other than this worker's GPU (``"cpu"``: pinned host
  memory, or another GPU) keeps the store off the GPU; loads are staged
  through a device ring and run on their own streams while the forward pass
  proceeds: ``wait_for_layer_load`` orders each layer's attention after its
  rows.  For any store, the load's status is checked in ``wait_for_save``
  rather than by blocking ``start_load_kv`` (``async_tier_load: false`` or
  ``MARATHON_VERIFY_LOAD=1`` restore the blocking load).

Paged layouts: the fused 4-D layouts the reference asserts (NHD/HND,
``:393-402``) and the 5-D split layouts of vLLM 0.22's FlashAttention
``(2, blocks, block_size, heads, head_size)`` and FlashInfer
``(blocks, 2, block_size, heads, head_size)``.  FP8 (e4m3) caches are
dequantised, rotated and requantised with each layer's K scale.

Failures are declined, never guessed at (the reference's rule,
``:104-109``), on both directions of the data path:

* a save the kernel refused (a bad slot, a store row out of range) is found
  from the step's status word, read back without stalling the forward pass;
  the session's store is truncated back to the start of that save on the
  worker, and the scheduler's mirror does the same when it receives the
  worker metadata (``build_connector_worker_meta`` ->
  ``update_connector_output``), so the next turn recomputes that span;
* a load that could not run (the store no longer holds the rows) or that the
  kernel refused is reported through ``get_block_ids_with_load_errors``, which
  makes vLLM recompute (or fail) those blocks instead of attending to them.
"""

from __future__ import annotations

import importlib
import importlib.util
import os
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import TYPE_CHECKING, Any

import torch
from vllm.distributed.kv_transfer.kv_connector.v1.base import (
    KVConnectorBase_V1,
    KVConnectorMetadata,
    KVConnectorRole,
)
from vllm.logger import init_logger

try:  # the worker -> scheduler channel (vLLM >= 0.11)
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorWorkerMetadata
except ImportError:  # pragma: no cover - older vLLM: failed saves stay worker-side
    KVConnectorWorkerMetadata = object

from . import _lib
from .shift_kernels import RopeShift, ShiftError, inv_freq as make_inv_freq, rope_shift, warmup
from .shift_store import (
    DEFAULT_STORE_TOKENS,
    SessionTable,
    ShiftStore,
    plan_load,
    plan_save,
    slots,
)
from .extent_store import ExtentStore
from .store_tier import DEFAULT_CHUNK_BYTES
from .worker import LoadJob, SaveJob, ShiftWorker

if TYPE_CHECKING:
    from vllm.config import VllmConfig
    from vllm.forward_context import ForwardContext
    from vllm.v1.core.kv_cache_manager import KVCacheBlocks
    from vllm.v1.core.sched.output import SchedulerOutput
    from vllm.v1.kv_cache_interface import KVCacheConfig
    from vllm.v1.request import Request

logger = init_logger("vllm.marathon_shift")

#: read every loaded span back and compare it with a torch fp32 re-rotation
#: (diagnostic, off by default; ``vllm_shift_connector.py:95-102``)
VERIFY_LOAD = os.environ.get("MARATHON_VERIFY_LOAD", "") not in ("", "0")
#: single-request multi-segment loads through a vLLM patched to honour a gap
#: plan (``vllm_shift_connector.py:104-110``); also ``"gapfill": true`` in
#: the connector's extra config
GAPFILL = os.environ.get("MARATHON_GAPFILL", "") not in ("", "0")
#: defer per-layer saves to wait_for_save and run them as one launch
BATCH_SAVE = os.environ.get("MARATHON_BATCH_SAVE", "") not in ("", "0")

# scheduler- and worker-side instances (possibly in different processes) all
# register here so `stats()` reports what is reachable from the caller
_STORES: list[ShiftStore] = []
_COUNTERS = ("hits", "misses", "evictions", "refusals", "loaded_token_layers",
             "saved_token_layers")


def stats() -> dict:
    """Store counters of every connector instance in this process, merged.

    Counters add up across instances; sizes (``used_tokens``, per-session
    tokens) are the largest any instance reports, because the scheduler's
    mirror and the worker's store describe the same sessions twice.  Same keys
    as the reference's ``stats()`` (``vllm_shift_connector.py:121-136``).
    """
    snaps = [store.stats() for store in _STORES]
    merged: dict[str, Any] = {k: sum(s[k] for s in snaps) for k in _COUNTERS}
    sessions: dict[str, int] = {}
    for snap in snaps:
        for name, tokens in snap["sessions"].items():
            sessions[name] = max(tokens, sessions.get(name, 0))
    merged["sessions"] = sessions
    merged["used_tokens"] = max((s["used_tokens"] for s in snaps), default=0)
    merged["budget_tokens"] = snaps[-1]["budget_tokens"] if snaps else 0
    return merged


def ulp(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Unit in the last place of ``dtype`` at each fp32 value of ``x``.

    ``2**(e - 1 - m)`` for ``|x|`` in ``[2**(e-1), 2**e)`` and ``m`` stored
    mantissa bits (7 bf16, 10 fp16, 23 fp32); the subnormal spacing
    ``tiny * eps`` below the normal range and at zero.
    """
    fi = torch.finfo(dtype)
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    _, e = torch.frexp(x.abs().to(torch.float32))
    step = torch.ldexp(torch.ones_like(x, dtype=torch.float32), e - 1 - mant)
    floor = torch.full_like(step, fi.smallest_normal * fi.eps)
    return torch.where(x == 0, floor, torch.maximum(step, floor))


@dataclass
class _Load:
    """One load: store rows ``[src_start, +length)`` -> positions ``[dst_start, +length)``."""

    session: str
    src_start: int
    delta: int
    dst_start: int
    length: int
    block_ids: list[int]
    block_size: int
    gen: int = -1  # extent-store mode: the generation whose keys are loaded

    @property
    def slots(self) -> torch.Tensor:
        """Flat destination slots, as the reference's ``_Load.slots`` carried them."""
        return slots(self.block_ids, self.dst_start, self.dst_start + self.length,
                     self.block_size)


@dataclass
class _Save:
    """One step's save: positions ``[dst_start, +length)`` -> the same store rows."""

    session: str
    dst_start: int
    length: int
    block_ids: list[int]
    block_size: int
    gen: int = -1  # extent-store mode: the generation computing these keys

    @property
    def slots(self) -> torch.Tensor:
        return slots(self.block_ids, self.dst_start, self.dst_start + self.length,
                     self.block_size)


@dataclass
class ShiftConnectorMetadata(KVConnectorMetadata):
    loads: list[_Load] = field(default_factory=list)
    saves: list[_Save] = field(default_factory=list)
    # extent-store mode: (session, gen, pos0, n) extents the view no longer uses
    releases: list[tuple[str, int, int, int]] = field(default_factory=list)


class _GenCover:
    """``covers`` of one generation of an :class:`ExtentStore`, for ``plan_load``."""

    def __init__(self, store: ExtentStore, gen: int) -> None:
        self.store, self.gen = store, gen

    def covers(self, session: str, start: int, n: int) -> bool:
        return self.store.locate(session, self.gen, start, n) is not None


@dataclass
class ShiftWorkerMetadata(KVConnectorWorkerMetadata):
    """Worker -> scheduler: store spans whose save did not land.

    ``truncate`` holds ``(session, pos)`` for the flat store (positions from
    ``pos`` on are forgotten), ``release`` holds ``(session, gen, pos0, n)``
    for the extent store.  The scheduler's mirror applies the same change, so
    its next ``plan_load`` declines rather than plan a load of rows that were
    never written.  With tensor parallelism every rank reports its own; the
    changes are idempotent, so the aggregate is the concatenation.
    """

    truncate: list[tuple[str, int]] = field(default_factory=list)
    release: list[tuple[str, int, int, int]] = field(default_factory=list)

    def aggregate(self, other: ShiftWorkerMetadata) -> ShiftWorkerMetadata:
        return ShiftWorkerMetadata(self.truncate + other.truncate,
                                   self.release + other.release)

    def __bool__(self) -> bool:
        return bool(self.truncate or self.release)


class GapHandoff:
    """The gap-fill hand-off to a vLLM patched to honour a non-prefix match.

    vLLM's connector API can only report externally supplied KV as a prefix.
    The reference's vLLM patch (``scripts/patch_vllm_gapfill.py``) changes
    that for one request: its scheduler ``take``s the plan a connector
    ``offer``ed on ``marathon.gapfill_channel`` and ``publish``es it, and its
    model runner overwrites the request's positions with ``active()``'s
    (``patch_vllm_gapfill.py:60-68``, ``:82-84``).  The plan itself is the
    reference's ``marathon.gapfill.plan_gaps`` (``src/marathon/gapfill.py:82-106``).
    Both are the reference's, consumed unchanged and imported by name: the
    patch reads exactly that channel module, so offering anywhere else would
    never reach it.

    The hand-off is available only when the channel and planner modules
    import and the installed vLLM carries the patch (its marker line in the
    scheduler and the model runner).  Otherwise the connector declines such a
    request (0 matched tokens): telling an unpatched vLLM that the filled
    spans are matched would make it treat them as one contiguous prefix and
    leave the gaps neither computed nor loaded.
    """

    PATCH_MARK = "# marathon: gapfill"
    PATCHED_FILES = ("v1/core/sched/scheduler.py", "v1/worker/gpu_model_runner.py")

    def __init__(self, channel: str = "marathon.gapfill_channel",
                 planner: str = "marathon.gapfill", require_patch: bool = True) -> None:
        self.channel_name, self.planner_name = channel, planner
        self.require_patch = require_patch
        self.channel = None
        self.plan_gaps = None
        self.why = ""
        self._resolved = False

    @classmethod
    def vllm_patched(cls) -> bool:
        """Whether the installed vLLM carries the gap-fill patch in both files."""
        spec = importlib.util.find_spec("vllm")
        if spec is None or not spec.submodule_search_locations:
            return False
        root = Path(next(iter(spec.submodule_search_locations)))
        try:
            return all(cls.PATCH_MARK in (root / f).read_text() for f in cls.PATCHED_FILES)
        except OSError:
            return False

    def ready(self) -> bool:
        """Resolve the channel, planner and patch once; True if the hand-off works."""
        if not self._resolved:
            self._resolved = True
            try:
                channel = importlib.import_module(self.channel_name)
                planner = importlib.import_module(self.planner_name)
                missing = [f for f in ("offer", "release") if not hasattr(channel, f)]
                if missing or not hasattr(planner, "plan_gaps"):
                    raise ImportError(f"{self.channel_name}/{self.planner_name} lack "
                                      f"{missing or ['plan_gaps']}")
            except ImportError as e:
                self.why = f"gap-fill channel unavailable ({e})"
                return False
            if self.require_patch and not self.vllm_patched():
                self.why = "the installed vLLM does not carry the gap-fill patch"
                return False
            self.channel, self.plan_gaps = channel, planner.plan_gaps
        return self.channel is not None

    def release(self, request_id: str) -> None:
        if self.channel is not None:
            self.channel.release(request_id)


def _rope_theta(hf) -> float:
    theta = getattr(hf, "rope_theta", None)
    if theta is None:
        params = getattr(hf, "rope_parameters", None) or getattr(hf, "rope_scaling", None) or {}
        theta = params.get("rope_theta") if isinstance(params, dict) else None
    return float(theta if theta is not None else 10000.0)


class MarathonShiftConnector(KVConnectorBase_V1):
    def __init__(self, vllm_config: VllmConfig, role: KVConnectorRole,
                 kv_cache_config: KVCacheConfig | None = None):
        super().__init__(vllm_config, role, kv_cache_config)
        self._bs = vllm_config.cache_config.block_size
        extra = self._kv_transfer_config.kv_connector_extra_config or {}
        budget = int(extra.get("store_tokens",
                               os.environ.get("MARATHON_STORE_TOKENS", DEFAULT_STORE_TOKENS)))
        device = str(extra.get("store_device", "cuda"))
        cap = int(extra.get("session_tokens", 0) or 0)
        # "window": the reference's flat per-session store; "extents": the
        # generation-tagged interval store (reuse without re-saving)
        self._extents = str(extra.get("store_mode", "window")) == "extents"
        if self._extents:
            self._store = ExtentStore(budget, device, allocate=(role == KVConnectorRole.WORKER))
        else:
            self._store = ShiftStore(budget, device, allocate=(role == KVConnectorRole.WORKER),
                                     session_cap=cap)
        _STORES.append(self._store)
        self._batch_save = bool(extra.get("batch_save", BATCH_SAVE))
        # loads from a store off the GPU overlap the forward pass, layer by layer
        self._async_tier = bool(extra.get("async_tier_load", True))
        # a step's save status is read back when it is ready ("deferred": the
        # forward pass is never stalled for it; it is waited for before any
        # later load) or at the end of the step ("sync")
        self._sync_save_check = str(extra.get("save_check", "deferred")) == "sync"
        self._gapfill = bool(extra.get("gapfill", GAPFILL))
        self._gap = GapHandoff(str(extra.get("gapfill_channel", "marathon.gapfill_channel")),
                               str(extra.get("gapfill_planner", "marathon.gapfill")),
                               bool(extra.get("gapfill_require_patch", True)))
        self._gap_declined = False  # logged once

        # scheduler side
        self._table = SessionTable()
        self._params: dict[str, dict[str, Any]] = {}
        self._plans: dict[str, tuple[int, int, int, int]] = {}
        self._multi: dict[str, list[dict]] = {}
        self._need_load: set[str] = set()
        self._blocks: dict[str, list[int]] = {}

        # worker side
        hf = vllm_config.model_config.hf_text_config
        head_dim = getattr(hf, "head_dim", None) or hf.hidden_size // hf.num_attention_heads
        rotary = int(head_dim * getattr(hf, "partial_rotary_factor", 1.0))
        self._inv_freq = make_inv_freq(rotary, _rope_theta(hf))
        self._rotary = rotary
        cache_dtype = str(getattr(vllm_config.cache_config, "cache_dtype", "auto"))
        self._fp8 = cache_dtype.startswith("fp8")
        # a store_device other than this worker's GPU ("cpu": pinned host memory) is
        # reached through staged copies of this many bytes per chunk
        chunk = int(extra.get("stage_chunk_bytes", DEFAULT_CHUNK_BYTES))
        self._worker = ShiftWorker(self._store, self._bs, self._inv_freq, fp8=self._fp8,
                                   chunk_bytes=chunk)
        self._kv: dict[str, torch.Tensor] = {}
        self._hnd: bool | None = None
        self._head_size: int | None = None
        self._rope: RopeShift | None = None
        self._pending_saves: list[tuple[str, torch.Tensor]] = []
        # save status: every save launch of a step ORs its rejected-token bits
        # into one device word; its copy is read once ready
        self._save_status: torch.Tensor | None = None
        self._step_saves: list[_Save] | None = None  # saves issued this step
        self._unchecked: list[tuple[torch.cuda.Event, torch.Tensor, list[_Save]]] = []
        self._failed = ShiftWorkerMetadata()  # for the scheduler's mirror
        self.save_failures = 0
        # loads: the queued load's jobs (status read at wait_for_save) and the
        # blocks of loads that did not land, for get_block_ids_with_load_errors
        self._queued_jobs: list[LoadJob] = []
        self._load_errors: set[int] = set()
        self.verify_mismatches = 0

    # ---------------------------------------------------------------- scheduler
    def on_new_request(self, request: Request) -> None:
        params = request.kv_transfer_params or {}
        self._params[request.request_id] = params
        session = params.get("session")
        if not session:
            return  # no session: pass-through, as if there were no connector
        if not self._table.acquire(request.request_id, str(session)):
            logger.warning(
                "shift: session %s already has an in-flight writer; request %s runs with no "
                "reuse (single writer per session)", session, request.request_id)

    def _accept_multi(self, request: Request, session: str, loads: list, num_computed: int):
        """Block-align and coverage-check every segment of a single-request load.

        A segment is dropped, never guessed at, when alignment leaves less than
        a block, when it lies inside vLLM's own prefix hit, or when the store no
        longer holds its source (``vllm_shift_connector.py:225-245``).
        """
        limit = (request.num_prompt_tokens - 1) // self._bs * self._bs
        floor = -(-num_computed // self._bs) * self._bs
        out = []
        for ld in loads:
            delta = int(ld["delta"])
            lo = max(-(-int(ld["dst_start"]) // self._bs) * self._bs, floor)
            hi = min(int(ld["dst_end"]), limit) // self._bs * self._bs
            if hi - lo < self._bs:
                continue
            if not self._cover(ld).covers(session, lo - delta, hi - lo):
                logger.warning("shift: gapfill dropping [%d,%d): store lost the source", lo, hi)
                continue
            out.append({"dst_start": lo, "dst_end": hi, "delta": delta,
                        "gen": int(ld.get("gen", -1))})
        return out

    def _cover(self, load: dict):
        """What answers coverage for ``load``: the store, or one generation of it."""
        if not self._extents:
            return self._store
        return _GenCover(self._store, int(load.get("gen", -1)))

    def get_num_new_matched_tokens(self, request: Request,
                                   num_computed_tokens: int) -> tuple[int | None, bool]:
        session = self._table.session_of(request.request_id)
        params = self._params.get(request.request_id) or {}

        multi = params.get("loads")
        if self._gapfill and session and multi and self._extents:
            # a gap-filled step computes scattered positions; saving its range
            # as one generation would tag loaded keys as fresh ones
            logger.warning("shift: the extent store does not take single-request "
                           "multi-segment loads; recomputing")
            return 0, False
        if self._gapfill and session and multi:
            if not self._gap.ready():
                # decline, never guess (vllm_shift_connector.py:104-109)
                if not self._gap_declined:
                    self._gap_declined = True
                    logger.warning("shift: declining multi-segment reuse: %s", self._gap.why)
                return 0, False
            accepted = self._accept_multi(request, session, multi, num_computed_tokens)
            if not accepted:
                return 0, False
            gp = self._gap.plan_gaps(accepted, self._bs, request.num_prompt_tokens,
                                     local_hit=num_computed_tokens)
            self._gap.channel.offer(request.request_id, gp.compute, gp.filled_tokens)
            self._multi[request.request_id] = accepted
            logger.info("shift: gapfill %d segments, %d/%d tokens filled, %d to compute",
                        len(accepted), gp.filled_tokens, gp.n_prompt, len(gp.compute))
            return max(gp.filled_tokens - num_computed_tokens, 0), False

        req = params.get("load")
        if self._extents and req and "gen" not in req:
            logger.warning("shift: extent store needs the load's generation; recomputing")
            return 0, False
        decision, why = plan_load(self._cover(req or {}), session, req, num_computed_tokens,
                                  request.num_prompt_tokens, self._bs)
        if decision is None:
            if session and req:
                logger.warning("shift: session %s declining reuse: %s", session, why)
            return 0, False
        self._plans[request.request_id] = (decision.lo, decision.hi, decision.delta,
                                           int(req.get("gen", -1)))
        return decision.hi - decision.lo, False

    def update_state_after_alloc(self, request: Request, blocks: KVCacheBlocks,
                                 num_external_tokens: int):
        if num_external_tokens > 0:
            self._need_load.add(request.request_id)

    def _plan_save(self, meta: ShiftConnectorMetadata, rid: str, lo: int, hi: int) -> None:
        """Record this step's save; ``"full"`` widens to ``[0, hi)`` once, then downgrades.

        (``vllm_shift_connector.py:296-330``: an edit turn rewrites the store in
        the new coordinates once; latching "full" would re-gather the whole
        prompt on every decode step.)
        """
        session = self._table.session_of(rid)
        blocks = self._blocks.get(rid)
        if not blocks:
            return
        params = self._params.get(rid) or {}
        if self._extents:
            # only what this step computed is saved, tagged with the turn's
            # generation; reused spans keep the rows of the turn that made them
            gen = params.get("gen")
            if not session or not params.get("save") or hi <= lo:
                return
            if gen is None or not self._store.save_extent(session, int(gen), lo, hi - lo):
                logger.warning("shift: session %s refused save of [%d,%d) (generation %s)",
                               session, lo, hi, gen)
                return
            meta.saves.append(_Save(session, lo, hi - lo, list(blocks), self._bs, int(gen)))
            return
        window = plan_save(self._store, session, params.get("save"), lo, hi)
        if window is None:
            if session and params.get("save") and hi > lo:
                logger.warning("shift: session %s refused save of [%d,%d)", session, lo, hi)
            return
        if params.get("save") == "full":
            params["save"] = True
        lo, hi = window
        meta.saves.append(_Save(session or "", lo, hi - lo, list(blocks), self._bs))

    def build_connector_meta(self, scheduler_output: SchedulerOutput):
        """The loads and saves of one scheduler step.

        A newly scheduled request brings its block table, its extent releases
        and (when ``get_num_new_matched_tokens`` planned a match) its loads; a
        running request may bring more blocks.  Either way the positions the
        step computes are its save candidates, planned in scheduling order --
        the order the worker replays them in, so both stores touch and evict
        sessions alike.
        """
        meta = ShiftConnectorMetadata()
        computing: list[tuple[str, int]] = []  # (request, first position computed)
        for req in scheduler_output.scheduled_new_reqs:
            self._blocks[req.req_id] = list(req.block_ids[0])
            self._admit(meta, req.req_id)
            computing.append((req.req_id, req.num_computed_tokens))
        cached = scheduler_output.scheduled_cached_reqs
        for rid, more, done in zip(cached.req_ids, cached.new_block_ids,
                                   cached.num_computed_tokens, strict=True):
            if more is not None:
                self._blocks.setdefault(rid, []).extend(more[0])
            computing.append((rid, done))
        for rid, lo in computing:
            self._plan_save(meta, rid, lo, lo + scheduler_output.num_scheduled_tokens[rid])
        for rid in scheduler_output.finished_req_ids:
            self._forget(rid)
        return meta

    def _admit(self, meta: ShiftConnectorMetadata, rid: str) -> None:
        """A request's first scheduled step: its releases and the loads planned for it."""
        session = self._table.session_of(rid) or ""
        if self._extents and session:
            for g, p0, n in (self._params.get(rid) or {}).get("release", ()):
                self._store.release(session, int(g), int(p0), int(n))
                meta.releases.append((session, int(g), int(p0), int(n)))
        if rid not in self._need_load:
            return
        self._need_load.discard(rid)
        table = self._blocks[rid]  # one block table, shared by all the request's segments
        if rid in self._multi:
            segments = [(s["dst_start"], s["dst_end"], s["delta"], s.get("gen", -1))
                        for s in self._multi[rid]]
        else:
            segments = [self._plans[rid]]
        for lo, hi, delta, gen in segments:
            meta.loads.append(_Load(session, lo - delta, delta, lo, hi - lo, list(table),
                                    self._bs, gen))

    def update_connector_output(self, connector_output) -> None:
        """Scheduler side: apply the workers' failed saves to the mirror store."""
        meta = getattr(connector_output, "kv_connector_worker_meta", None)
        if isinstance(meta, ShiftWorkerMetadata):
            self._apply_failed(meta)

    def _apply_failed(self, meta: ShiftWorkerMetadata) -> None:
        for session, pos in meta.truncate:
            self._store.truncate(session, pos)
        for session, gen, pos0, n in meta.release:
            self._store.release(session, gen, pos0, n)

    def _forget(self, rid: str) -> None:
        """Drop everything held for a finished request (idempotent)."""
        for held in (self._multi, self._blocks, self._params, self._plans):
            held.pop(rid, None)
        self._need_load.discard(rid)
        self._gap.release(rid)
        self._table.release(rid)

    def request_finished(self, request: Request, block_ids: list[int]):
        self._forget(request.request_id)
        logger.info("shift: store %s", self._store.stats())
        return False, None

    # ------------------------------------------------------------------ worker
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]):
        self._kv = kv_caches
        first = next(iter(kv_caches.values()))
        shape = tuple(first.shape)
        if first.dim() == 4:
            from .paged import detect_hnd

            self._hnd = detect_hnd(shape, self._bs)
            self._head_size = shape[3] // 2
            self._worker.layout = "hnd" if self._hnd else "nhd"
        elif first.dim() == 5:
            self._hnd = False
            self._head_size = shape[4]
            self._worker.layout = "split" if shape[0] == 2 else "split_blocks"
        else:
            raise AssertionError(f"expected a 4-D fused or 5-D split KV layout, got {shape}")
        # an unsupported geometry fails here, at registration, as the
        # reference's warmup did (vllm_shift_connector.py:405)
        warmup(first, self._bs, bool(self._hnd), rotary=self._rotary,
               layout=self._worker.layout, fp8=self._fp8)
        if first.is_cuda:
            self._worker.register(kv_caches)
        logger.info("marathon shift connector: %d layers, kv shape %s, layout %s, store %d tok",
                    len(kv_caches), shape, self._worker.layout, self._store.budget)

    def _shift(self, delta: int, device) -> RopeShift:
        """Rotation tables of one delta (reference API; the batched path builds its own)."""
        if self._rope is None or self._rope.delta != delta or self._rope.cos.device != device:
            self._rope = rope_shift(delta, self._head_size, self._inv_freq, device)
        return self._rope

    def _k_scales(self, forward_context) -> torch.Tensor | None:
        if not self._fp8:
            return None
        layers = getattr(forward_context, "no_compile_layers", {}) or {}
        vals = []
        for name in self._worker.layers.names:
            s = getattr(layers.get(name), "_k_scale", None)
            vals.append(float(s) if s is not None else 1.0)
        return torch.tensor(vals, dtype=torch.float32)

    def start_load_kv(self, forward_context: ForwardContext, **kwargs: Any) -> None:
        meta = self._get_connector_metadata()
        if not isinstance(meta, ShiftConnectorMetadata):
            return
        for session, g, p0, n in meta.releases:  # mirrors the scheduler's releases
            self._store.release(session, g, p0, n)
        if not meta.loads:
            return
        if not self._worker.registered:
            caches = {
                n: layer.kv_cache[forward_context.virtual_engine]
                if isinstance(getattr(layer, "kv_cache", None), list) else layer.kv_cache
                for n, layer in forward_context.no_compile_layers.items()
                if getattr(layer, "kv_cache", None) is not None
            }
            self.register_kv_caches(caches)
        # a save of an earlier step that the kernel refused must be known (and
        # its span forgotten) before any load reads those rows
        self._poll_saves(block=True)
        if self._fp8:
            self._worker.k_scales = self._k_scales(forward_context)
            if self._worker.k_scales is not None:
                self._worker.k_scales = self._worker.k_scales.to(self._worker.layers.device)
        if self._extents:
            jobs, lost = self._extent_load_jobs(meta.loads)
            self._note_load_errors(lost)
        else:
            jobs = [LoadJob(ld.session, ld.src_start, ld.delta, ld.dst_start, ld.length,
                            block_ids=ld.block_ids) for ld in meta.loads]
        # the load is queued and its status checked in wait_for_save: a store
        # off the GPU streams in layer by layer behind the forward pass
        # (wait_for_layer_load orders each layer's attention after its rows);
        # a device store's load runs on the forward pass's own stream, ahead
        # of it, without the host waiting for it as the reference did
        queued = self._async_tier and not VERIFY_LOAD
        t0 = time.perf_counter()
        try:
            done = self._worker.load(jobs, check=True, asynchronous=queued)
        except ShiftError as e:  # a synchronous load the kernel refused
            logger.error("shift: load failed (%s); its blocks are reported for recompute", e)
            self._note_load_errors(jobs)
            return
        # a job whose rows the store no longer holds stops the batch there
        self._note_load_errors(jobs[len(done):])
        if queued:
            self._queued_jobs = list(done)
        ms = (time.perf_counter() - t0) * 1e3
        geo = self._worker.layers.geometry
        moved = sum(j.length for j in done) * len(self._worker.layers) * geo.heads * \
            2 * geo.head_size * geo.elem_bytes
        for j in done:
            logger.info("shift: session %s loaded %d tokens x %d layers from store[%d:%d], "
                        "delta=%d", j.session, j.length, len(self._worker.layers), j.src_start,
                        j.src_start + j.length, j.delta)
        if queued:
            logger.info("shift: %d load(s) queued from the %s store (%.2f MB, %.2f ms "
                        "to queue)", len(done), self._store.device, moved / 2**20, ms)
        else:
            logger.info("shift: %d load(s) in one launch, copy_ms=%.2f (%.2f MB, %.1f GB/s)",
                        len(done), ms, moved / 2**20, moved / 2**30 / max(ms / 1e3, 1e-9))
        if VERIFY_LOAD and not self._extents:
            for j in done:
                if not self._verify(j):
                    self._note_load_errors([j])
        logger.info("shift: store %s", self._store.stats())

    def _note_load_errors(self, jobs) -> None:
        """Report the destination blocks of loads that did not land.

        vLLM reads them through ``get_block_ids_with_load_errors`` and
        recomputes those blocks (or fails the request, per its
        ``kv_load_failure_policy``) instead of attending to stale KV.
        """
        for j in jobs:
            if j.block_ids is None or j.length <= 0:
                continue
            lo = j.dst_start // self._bs
            hi = -(-(j.dst_start + j.length) // self._bs)
            self._load_errors.update(int(b) for b in list(j.block_ids)[lo:hi])

    def get_block_ids_with_load_errors(self) -> set[int]:
        out, self._load_errors = self._load_errors, set()
        return out

    def _extent_load_jobs(self, loads: list[_Load]) -> tuple[list[LoadJob], list[_Load]]:
        """A load of generation ``gen``'s positions as one job per store extent,
        plus the loads whose rows the store no longer holds."""
        jobs, lost = [], []
        for ld in loads:
            where = self._store.locate(ld.session, ld.gen, ld.src_start, ld.length, count=False)
            if where is None:
                logger.error("shift: session %s generation %d lost [%d,%d); load skipped",
                             ld.session, ld.gen, ld.src_start, ld.src_start + ld.length)
                lost.append(ld)
                continue
            for p0, n, row in where:
                jobs.append(LoadJob(ld.session, p0, ld.delta, p0 + ld.delta, n,
                                    block_ids=ld.block_ids, store_start=row))
        return jobs, lost

    def _extent_save_jobs(self, save: _Save) -> list[SaveJob]:
        """This step's fresh positions as one job per extent (the scheduler's allocation)."""
        return [SaveJob(save.session, p0, n, block_ids=save.block_ids, store_start=row)
                for p0, n, row in self._store.save_extent(save.session, save.gen,
                                                         save.dst_start, save.length)]

    def _verify(self, job: LoadJob) -> bool:
        """Read a loaded span back and check it against the torch fp32 rotation.

        The reference's diagnostic (``vllm_shift_connector.py:444-479``) with a
        pass/fail bar instead of a logged difference: V and any non-rotary
        tail bit for bit, and every rotated K element within one unit in the
        last place (of the cache dtype) of ``k*cos + rotate_half(k)*sin``
        evaluated by torch in fp32 with the reference's own tables -- torch's
        fp32 cos/sin of ``fp32(delta) * inv_freq`` on the cache's device, as
        its ``rope_shift`` builds them (``shift_kernels.py:68-84``).  Plain
        torch operations on copies of the store rows and the paged rows: it
        shares nothing with the kernel.  Returns False (and logs an error) on
        any mismatch.
        """
        geo = self._worker.layers.geometry
        cache_dtype = self._worker.layers.tensors[0].dtype
        if cache_dtype not in (torch.bfloat16, torch.float16, torch.float32):
            logger.warning("shift-verify: %s cache unsupported; skipped", cache_dtype)
            return True
        d, rot = geo.head_size, self._rotary
        h = rot // 2
        sl = job.host_slots(self._bs)
        bits = {2: torch.int16, 4: torch.int32}[geo.elem_bytes]
        ok = True
        for name, kv in zip(self._worker.layers.names, self._worker.layers.tensors, strict=True):
            row = self._store.read(job.session, name, job.row, job.length)
            if row is None:
                continue
            row = row.to(kv.device)  # a host or peer store tier
            ang = float(job.delta) * self._inv_freq.to(kv.device, torch.float32)
            cos, sin = torch.cat((ang, ang)).cos(), torch.cat((ang, ang)).sin()
            b, o = (sl // self._bs).to(kv.device), (sl % self._bs).to(kv.device)
            if geo.kind == "hnd":
                got = kv[b, :, o]
            elif geo.kind == "nhd":
                got = kv[b, o]
            else:
                kk, vv = (kv[0], kv[1]) if geo.kind == "split" else (kv[:, 0], kv[:, 1])
                got = torch.cat((kk[b, o], vv[b, o]), -1)
            kf = row[..., :rot].float()
            want = kf * cos + torch.cat((-kf[..., h:], kf[..., :h]), -1) * sin
            k_off = (got[..., :rot].float() - want).abs() > ulp(want, cache_dtype)
            exact = got[..., rot:].view(bits) != row[..., rot:].view(bits)
            n_k, n_x = int(k_off.sum()), int(exact.sum())
            if n_k or n_x:
                ok = False
                logger.error("shift-verify: layer=%s delta=%d n=%d: %d K elements beyond one "
                             "ulp of the fp32 rotation, %d V/tail elements not bit-equal",
                             name, job.delta, job.length, n_k, n_x)
            else:
                logger.info("shift-verify: layer=%s delta=%d n=%d ok", name, job.delta,
                            job.length)
        if not ok:
            self.verify_mismatches += 1
        return ok

    def wait_for_layer_load(self, layer_name: str) -> None:
        if self._worker.pending is not None and layer_name in self._worker.layers.index:
            self._worker.wait_layer(layer_name)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata, **kw):
        meta = self._get_connector_metadata()
        if not isinstance(meta, ShiftConnectorMetadata) or not meta.saves:
            return
        if not self._worker.registered:
            self.register_kv_caches({layer_name: kv_layer})
        if layer_name not in self._worker.layers.index:
            # a cache that was not registered up front (lazy per-layer discovery)
            caches = dict(zip(self._worker.layers.names, self._worker.layers.tensors,
                              strict=True))
            caches[layer_name] = kv_layer
            self._worker.register(caches)
        if self._batch_save:
            self._pending_saves.append((layer_name, kv_layer))
            return
        self._save_layers([layer_name], meta)

    def _save_layers(self, names: list[str], meta: ShiftConnectorMetadata) -> None:
        jobs, issued = [], []
        if self._extents:
            for save in meta.saves:
                jobs.extend(self._extent_save_jobs(save))
                issued.append(save)
            self._issue_saves(jobs, names, issued)
            return
        for save in meta.saves:
            # mirrors the scheduler's reserve for this step; idempotent across layers
            if not self._store.reserve(save.session, save.dst_start, save.length):
                continue
            jobs.append(SaveJob(save.session, save.dst_start, save.length,
                                block_ids=save.block_ids))
            issued.append(save)
        self._issue_saves(jobs, names, issued)

    def _issue_saves(self, jobs: list[SaveJob], names: list[str], saves: list[_Save]) -> None:
        """Launch a save; its rejected-token bits join the step's status word."""
        if not jobs:
            return
        if self._step_saves is None:  # the step's first save: a fresh status word
            if self._save_status is None:
                self._save_status = torch.zeros(4, dtype=torch.int32,
                                                device=self._worker.layers.device)
            else:
                self._save_status.zero_()
            self._step_saves = list(saves)
        self._worker.save(jobs, names, check=False, err=self._save_status.data_ptr())

    def wait_for_save(self):
        # this step's queued load: the stream waits for it, the host reads its status
        try:
            self._worker.finish_pending()
        except ShiftError as e:
            logger.error("shift: load failed (%s); its blocks are reported for recompute", e)
            self._note_load_errors(self._queued_jobs)
        self._queued_jobs = []
        if self._pending_saves:
            meta = self._get_connector_metadata() if self.has_connector_metadata() else None
            names = [n for n, _ in self._pending_saves]
            self._pending_saves = []
            if isinstance(meta, ShiftConnectorMetadata) and meta.saves:
                # one launch per run of consecutive layers (normally: all of them)
                order = sorted(names, key=self._worker.layers.index.__getitem__)
                group: list[str] = []
                for n in order:
                    if group and self._worker.layers.index[n] != \
                            self._worker.layers.index[group[-1]] + 1:
                        self._save_layers(group, meta)
                        group = []
                    group.append(n)
                if group:
                    self._save_layers(group, meta)
        self._close_step_saves()

    def _close_step_saves(self) -> None:
        """Queue the read-back of this step's save status (read when it is ready)."""
        if self._step_saves is None:
            return
        word = torch.empty(1, dtype=torch.int32, pin_memory=True)
        word.copy_(self._save_status[:1], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._unchecked.append((ev, word, self._step_saves))
        self._step_saves = None
        self._poll_saves(block=self._sync_save_check)

    def _poll_saves(self, block: bool) -> None:
        """Read the save statuses that are ready (all of them when ``block``)."""
        while self._unchecked:
            ev, word, saves = self._unchecked[0]
            if not block and not ev.query():
                return
            ev.synchronize()
            self._unchecked.pop(0)
            bits = int(word[0])
            if bits:
                self._saves_failed(saves, bits)

    def _saves_failed(self, saves: list[_Save], bits: int) -> None:
        """Forget the spans of a refused save here and, through the worker
        metadata, in the scheduler's mirror: the next turn recomputes them."""
        self.save_failures += 1
        logger.error("shift: the save kernel rejected tokens (%s); dropping %d stored span(s) "
                     "so later turns recompute them", _lib.describe_bits(bits), len(saves))
        for sv in saves:
            if self._extents:
                self._store.release(sv.session, sv.gen, sv.dst_start, sv.length)
                self._failed.release.append((sv.session, sv.gen, sv.dst_start, sv.length))
            else:
                self._store.truncate(sv.session, sv.dst_start)
                self._failed.truncate.append((sv.session, sv.dst_start))

    def build_connector_worker_meta(self):
        """Failed saves for the scheduler's mirror (None when there are none)."""
        self._poll_saves(block=False)
        if not self._failed:
            return None
        out, self._failed = self._failed, ShiftWorkerMetadata()
        return out
