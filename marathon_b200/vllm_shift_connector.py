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
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any

import torch
from vllm.distributed.kv_transfer.kv_connector.v1.base import (
    KVConnectorBase_V1,
    KVConnectorMetadata,
    KVConnectorRole,
)
from vllm.logger import init_logger

from . import gapfill
from .shift_kernels import RopeShift, inv_freq as make_inv_freq, rope_shift
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
#: plan (``vllm_shift_connector.py:104-110``)
GAPFILL = os.environ.get("MARATHON_GAPFILL", "") not in ("", "0")
#: defer per-layer saves to wait_for_save and run them as one launch
BATCH_SAVE = os.environ.get("MARATHON_BATCH_SAVE", "") not in ("", "0")

# scheduler- and worker-side instances (possibly in different processes) all
# register here so `stats()` reports what is reachable from the caller
_STORES: list[ShiftStore] = []
_COUNTERS = ("hits", "misses", "evictions", "refusals", "loaded_token_layers",
             "saved_token_layers")


def stats() -> dict:
    """Merged store counters across the connector instances of this process."""
    out: dict[str, Any] = dict.fromkeys(_COUNTERS, 0)
    out.update(sessions={}, used_tokens=0, budget_tokens=0)
    for store in _STORES:
        s = store.stats()
        out["budget_tokens"] = s["budget_tokens"]
        out["used_tokens"] = max(out["used_tokens"], s["used_tokens"])
        for name, filled in s["sessions"].items():
            out["sessions"][name] = max(out["sessions"].get(name, 0), filled)
        for k in _COUNTERS:
            out[k] += s[k]
    return out


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
        if GAPFILL and session and multi and self._extents:
            # a gap-filled step computes scattered positions; saving its range
            # as one generation would tag loaded keys as fresh ones
            logger.warning("shift: the extent store does not take single-request "
                           "multi-segment loads; recomputing")
            return 0, False
        if GAPFILL and session and multi:
            accepted = self._accept_multi(request, session, multi, num_computed_tokens)
            if not accepted:
                return 0, False
            gp = gapfill.plan_gaps(accepted, self._bs, request.num_prompt_tokens,
                                   local_hit=num_computed_tokens)
            gapfill.offer(request.request_id, gp.compute, gp.filled_tokens)
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
        meta = ShiftConnectorMetadata()
        for req in scheduler_output.scheduled_new_reqs:
            rid = req.req_id
            self._blocks[rid] = list(req.block_ids[0])
            session = self._table.session_of(rid) or ""
            if self._extents and session:
                for g, p0, n in (self._params.get(rid) or {}).get("release", ()):
                    self._store.release(session, int(g), int(p0), int(n))
                    meta.releases.append((session, int(g), int(p0), int(n)))
            if rid in self._need_load and rid in self._multi:
                table = list(self._blocks[rid])  # one block table shared by the segments
                for seg in self._multi[rid]:
                    n = seg["dst_end"] - seg["dst_start"]
                    meta.loads.append(_Load(session, seg["dst_start"] - seg["delta"],
                                            seg["delta"], seg["dst_start"], n, table, self._bs,
                                            seg.get("gen", -1)))
                self._need_load.discard(rid)
            elif rid in self._need_load:
                lo, hi, delta, gen = self._plans[rid]
                meta.loads.append(_Load(session, lo - delta, delta, lo, hi - lo,
                                        list(self._blocks[rid]), self._bs, gen))
                self._need_load.discard(rid)
            lo = req.num_computed_tokens
            self._plan_save(meta, rid, lo, lo + scheduler_output.num_scheduled_tokens[rid])

        cached = scheduler_output.scheduled_cached_reqs
        for i, rid in enumerate(cached.req_ids):
            new_blocks = cached.new_block_ids[i]
            if new_blocks is not None:
                self._blocks.setdefault(rid, []).extend(new_blocks[0])
            lo = cached.num_computed_tokens[i]
            self._plan_save(meta, rid, lo, lo + scheduler_output.num_scheduled_tokens[rid])

        for rid in scheduler_output.finished_req_ids:
            self._forget(rid)
        return meta

    def _forget(self, rid: str) -> None:
        gapfill.release(rid)
        self._multi.pop(rid, None)
        self._blocks.pop(rid, None)
        self._params.pop(rid, None)
        self._plans.pop(rid, None)
        self._need_load.discard(rid)
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
        if self._fp8:
            self._worker.k_scales = self._k_scales(forward_context)
            if self._worker.k_scales is not None:
                self._worker.k_scales = self._worker.k_scales.to(self._worker.layers.device)
        if self._extents:
            jobs = self._extent_load_jobs(meta.loads)
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
        done = self._worker.load(jobs, check=True, asynchronous=queued)
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
                self._verify(j)
        logger.info("shift: store %s", self._store.stats())

    def _extent_load_jobs(self, loads: list[_Load]) -> list[LoadJob]:
        """A load of generation ``gen``'s positions as one job per store extent."""
        jobs = []
        for ld in loads:
            where = self._store.locate(ld.session, ld.gen, ld.src_start, ld.length, count=False)
            if where is None:
                logger.error("shift: session %s generation %d lost [%d,%d); load skipped",
                             ld.session, ld.gen, ld.src_start, ld.src_start + ld.length)
                continue
            for p0, n, row in where:
                jobs.append(LoadJob(ld.session, p0, ld.delta, p0 + ld.delta, n,
                                    block_ids=ld.block_ids, store_start=row))
        return jobs

    def _extent_save_jobs(self, save: _Save) -> list[SaveJob]:
        """This step's fresh positions as one job per extent (the scheduler's allocation)."""
        return [SaveJob(save.session, p0, n, block_ids=save.block_ids, store_start=row)
                for p0, n, row in self._store.save_extent(save.session, save.gen,
                                                         save.dst_start, save.length)]

    def _verify(self, job: LoadJob) -> None:
        """Read a loaded span back and compare it with a torch fp32 re-rotation."""
        if self._rotary != self._head_size:
            logger.warning("shift-verify: partial rotary (%d of %d) unsupported; skipped",
                           self._rotary, self._head_size)
            return
        geo = self._worker.layers.geometry
        d = geo.head_size
        sl = job.host_slots(self._bs)
        for name, kv in zip(self._worker.layers.names, self._worker.layers.tensors, strict=True):
            row = self._store.read(job.session, name, job.src_start, job.length)
            if row is None:
                continue
            row = row.to(kv.device)  # a host or peer store tier
            sh = self._shift(job.delta, kv.device)
            kf = row[..., :d].float()
            h = d // 2
            want_k = kf * sh.emb_cos + torch.cat((-kf[..., h:], kf[..., :h]), -1) * sh.emb_sin
            blk, off = (sl // self._bs).to(kv.device), (sl % self._bs).to(kv.device)
            if geo.kind == "hnd":
                got = kv[blk, :, off]
            elif geo.kind == "nhd":
                got = kv[blk, off]
            else:
                kk, vv = (kv[0], kv[1]) if geo.kind == "split" else (kv[:, 0], kv[:, 1])
                got = torch.cat((kk[blk, off], vv[blk, off]), -1)
            want = torch.cat((want_k, row[..., d:].float()), -1)
            diff = (got.float() - want).abs()
            logger.info("shift-verify: layer=%s delta=%d n=%d max_abs=%.4g max_rel=%.4g", name,
                        job.delta, job.length, float(diff.max()),
                        float(diff.max() / want.abs().max().clamp_min(1e-6)))

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
        jobs = []
        if self._extents:
            for save in meta.saves:
                jobs.extend(self._extent_save_jobs(save))
            if jobs:
                self._worker.save(jobs, names, check=False)
            return
        for save in meta.saves:
            # mirrors the scheduler's reserve for this step; idempotent across layers
            if not self._store.reserve(save.session, save.dst_start, save.length):
                continue
            jobs.append(SaveJob(save.session, save.dst_start, save.length,
                                block_ids=save.block_ids))
        if jobs:
            self._worker.save(jobs, names, check=False)

    def wait_for_save(self):
        self._worker.finish_pending()  # this step's queued load: wait, check its status
        if not self._pending_saves:
            return
        meta = self._get_connector_metadata() if self.has_connector_metadata() else None
        names = [n for n, _ in self._pending_saves]
        self._pending_saves = []
        if not isinstance(meta, ShiftConnectorMetadata) or not meta.saves:
            return
        # one launch per run of consecutive layers (normally: all of them)
        order = sorted(names, key=self._worker.layers.index.__getitem__)
        group: list[str] = []
        for n in order:
            if group and self._worker.layers.index[n] != self._worker.layers.index[group[-1]] + 1:
                self._save_layers_batched(group, meta)
                group = []
            group.append(n)
        if group:
            self._save_layers_batched(group, meta)

    def _save_layers_batched(self, names: list[str], meta: ShiftConnectorMetadata) -> None:
        if self._extents:
            self._save_layers(names, meta)
            return
        jobs = []
        for save in meta.saves:
            if not self._store.reserve(save.session, save.dst_start, save.length):
                continue
            jobs.append(SaveJob(save.session, save.dst_start, save.length,
                                block_ids=save.block_ids))
        if jobs:
            self._worker.save(jobs, names, check=False)
