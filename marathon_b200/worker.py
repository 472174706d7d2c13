"""Worker side of the shift connector, independent of vLLM's plumbing.

:class:`ShiftWorker` is what ``MarathonShiftConnector`` runs on a worker: it
holds the registered paged caches and the session store, and turns one step's
loads (or saves) into ONE native launch over every load x every layer.  The
reference ran one Triton launch per layer per load, preceded by a
``ShiftStore.read`` and a slot transfer per layer
(``src/marathon/vllm_shift_connector.py:495-518``); here the decisions are the
same (``ShiftStore`` bookkeeping, counters and LRU touches per layer) but the
bytes move in a single persistent kernel, and the request's block table rides
to the device inside the batch's single descriptor copy instead of a per-token
slot tensor.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import numpy as np
import torch

from .paged import KVLayers
from .shift_kernels import Launcher, RunSpec, ShiftError
from .shift_store import ShiftStore, slots as host_slots
from .store_tier import DEFAULT_CHUNK_BYTES, StagedLoad, StagedMover, is_staged

logger = logging.getLogger("vllm.marathon_shift")


@dataclass
class LoadJob:
    """One load: store ``[src_start, +length)`` -> logical ``[dst_start, +length)``.

    ``store_start`` names the first store row when rows are not addressed by
    position (an :class:`~marathon_b200.extent_store.ExtentStore`); by
    default it is ``src_start``.
    """

    session: str
    src_start: int
    delta: int
    dst_start: int
    length: int
    block_ids: list[int] | np.ndarray | None = None
    slots: torch.Tensor | None = None  # alternative to block_ids: flat slots
    store_start: int | None = None

    @property
    def row(self) -> int:
        return self.src_start if self.store_start is None else self.store_start

    def host_slots(self, block_size: int) -> torch.Tensor:
        if self.slots is not None:
            return self.slots.cpu()
        return host_slots(list(self.block_ids), self.dst_start, self.dst_start + self.length,
                          block_size)


@dataclass
class SaveJob:
    """One save: logical positions ``[dst_start, +length)`` -> the same store rows
    (or the rows from ``store_start``, for an extent store)."""

    session: str
    dst_start: int
    length: int
    block_ids: list[int] | np.ndarray | None = None
    slots: torch.Tensor | None = None
    store_start: int | None = None

    @property
    def row(self) -> int:
        return self.dst_start if self.store_start is None else self.store_start


def _run(row: int, store_start: int, length: int, delta: int, block_ids, slots, paged_start,
         tables: dict):
    """A RunSpec; jobs that share one block-table object share one converted table."""
    if slots is not None:
        return RunSpec(row, store_start, length, delta, slots=slots)
    key = id(block_ids)
    bt = tables.get(key)
    if bt is None:
        bt = tables[key] = np.asarray(block_ids, np.int32)
    return RunSpec(row, store_start, length, delta, block_table=bt, paged_start=paged_start)


class ShiftWorker:
    """Registered caches + store; batched native load and save."""

    def __init__(
        self,
        store: ShiftStore,
        block_size: int,
        inv_freq: torch.Tensor,
        *,
        layout: str | None = None,
        fp8: bool = False,
        k_scales: torch.Tensor | None = None,
        chunk_bytes: int = DEFAULT_CHUNK_BYTES,
    ) -> None:
        self.store = store
        self.block_size = int(block_size)
        self.inv_cpu = inv_freq.to(torch.float32)
        self.layout = layout
        self.fp8 = fp8
        self.k_scales = k_scales
        self.layers: KVLayers | None = None
        self.launcher: Launcher | None = None
        self.inv: torch.Tensor | None = None
        # a store in host memory or on another GPU is reached by staged copies
        self.chunk_bytes = int(chunk_bytes)
        self.mover: StagedMover | None = None
        self.pending: StagedLoad | None = None  # an asynchronous load in flight

    @property
    def registered(self) -> bool:
        return self.layers is not None

    def register(self, kv_caches: dict[str, torch.Tensor]) -> KVLayers:
        self.layers = KVLayers(kv_caches, self.block_size, self.layout, fp8=self.fp8)
        self._name_set = frozenset(self.layers.names)
        self.launcher = Launcher(self.layers)
        self.inv = self.inv_cpu.to(self.layers.device)
        if is_staged(self.store.device, self.layers.device):
            self.mover = StagedMover(self.launcher, self.chunk_bytes)
            peer = torch.device(self.store.device)
            if peer.type == "cuda":
                self.mover.enable_peer(peer.index)
        if self.k_scales is not None:
            self.k_scales = self.k_scales.to(self.layers.device, torch.float32)
        return self.layers

    # ---------------------------------------------------------------- load
    def load(self, jobs: list[LoadJob], *, check: bool = True,
             asynchronous: bool = False) -> list[LoadJob]:
        """Every job x every layer in one launch.  Returns the jobs that were issued.

        A job whose rows are not all held (evicted, truncated, a layer never
        saved) stops the batch there, as the reference's load loop returned on
        the first missing layer (``vllm_shift_connector.py:506-513``): jobs
        before it are loaded, it and later ones are not.

        ``asynchronous``: return once the load is queued, with its status
        checked later by ``finish_pending``.  A store off the GPU is staged on
        the mover's own streams (``wait_layer`` orders a layer's consumers
        after its rows); a device store's load is queued on the current
        stream, so later work on that stream is ordered after it anyway and
        only the host-side status check is deferred -- to ``finish_pending``
        or to the next asynchronous ``load``, which packs and queues its own
        batch first, so a caller issuing loads back to back keeps the GPU busy
        while the host prepares the next one.
        """
        if not jobs:
            return []
        if self.launcher is None:
            raise ShiftError("no KV caches registered")
        prev = None
        if (asynchronous and self.mover is None and self.pending is not None
                and self.pending.same_stream):
            prev, self.pending = self.pending, None  # checked once this batch is queued
        else:
            self.finish_pending()
        try:
            return self._load(jobs, check, asynchronous)
        finally:
            if prev is not None:
                prev.check()

    def _load(self, jobs: list[LoadJob], check: bool, asynchronous: bool) -> list[LoadJob]:
        names = self.layers.names
        name_set = self._name_set
        accepted: list[LoadJob] = []
        for job in jobs:
            missing = self.store.loadable(job.session, names, job.row, job.length, name_set)
            if missing is not None:
                logger.error("shift: session %s has no stored KV for %s; load skipped",
                             job.session, missing)
                break
            self.store.mark_loaded(job.session, names, job.length)
            accepted.append(job)
        if not accepted:
            return []
        rows: dict[str, int] = {}
        runs = []
        tables: dict = {}
        for job in accepted:
            row = rows.setdefault(job.session, len(rows))
            runs.append(_run(row, job.row, job.length, job.delta, job.block_ids, job.slots,
                             job.dst_start, tables))
        view = self.store.view(list(rows), names)
        if self.mover is not None and asynchronous:
            self.pending = self.mover.load_async(runs, view, self.inv, k_scales=self.k_scales)
            return accepted
        if asynchronous:
            self.pending = self._queue_load(runs, view)
            return accepted
        mover = self.mover or self.launcher
        mover.load(runs, view, self.inv, k_scales=self.k_scales, check=check)
        return accepted

    def _queue_load(self, runs, view) -> StagedLoad:
        """One launch on the current stream; its status word is copied back
        asynchronously, off that stream, and read in ``finish_pending``."""
        la = self.launcher
        p = la.prepare_load(runs, view, self.inv, k_scales=self.k_scales)
        la.launch(p)
        la.finish(p, False)
        done = torch.cuda.Event()
        done.record(p.stream)
        errs = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        copied = la.staging.copy_err_after(p.slot, errs, done)
        return StagedLoad([done] * len(self.layers), copied, errs, 1, same_stream=True)

    def wait_layer(self, name: str) -> None:
        """Order the current stream after layer ``name`` of a pending staged load."""
        if self.pending is not None:
            self.pending.wait_layer(self.layers.index[name])

    def finish_pending(self) -> None:
        """Complete a pending load: the current stream waits for all of it,
        the host checks its status (raises :class:`ShiftError` on rejected tokens)."""
        job, self.pending = self.pending, None
        if job is not None:
            job.wait_all()
            job.check()

    # ---------------------------------------------------------------- save
    def save(self, jobs: list[SaveJob], layer_names: list[str] | None = None, *,
             check: bool = True, err: int | None = None) -> int:
        """Gather ``jobs`` out of the paged caches of ``layer_names`` into the store.

        The layers must be consecutive in registration order (one launch covers
        a contiguous range); the store rows must already be reserved.  Returns
        the number of token-layers written.  ``check`` waits and raises on
        rejected tokens; ``err`` (a device address, with ``check=False``) makes
        the kernels OR their rejected-token bits into that word instead, for a
        caller that reads one status per step.
        """
        if not jobs:
            return 0
        if self.launcher is None:
            raise ShiftError("no KV caches registered")
        if self.pending is not None:
            # the saved rows may be ones the pending load is still writing
            self.pending.wait_all()
        names = layer_names if layer_names is not None else self.layers.names
        idx = [self.layers.index[n] for n in names]
        first = idx[0]
        if idx != list(range(first, first + len(idx))):
            raise ShiftError("a batched save covers consecutive layers only")
        geo = self.layers.geometry
        dtype = self.layers.tensors[0].dtype
        rows: dict[str, int] = {}
        runs = []
        tables: dict = {}
        for job in jobs:
            if not self.store.ensure_layers(job.session, names, geo.heads, 2 * geo.head_size,
                                            dtype):
                continue
            if job.row + job.length > self.store.capacity(job.session):
                continue
            row = rows.setdefault(job.session, len(rows))
            runs.append(_run(row, job.row, job.length, 0, job.block_ids, job.slots,
                             job.dst_start, tables))
        if not runs:
            return 0
        view = self.store.view(list(rows), names)
        mover = self.mover or self.launcher
        mover.save(runs, view, first_layer=first, n_layers=len(names), check=check, err=err)
        done = sum(r.length for r in runs)
        self.store.mark_saved(done, len(names))
        return done * len(names)
