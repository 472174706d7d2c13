"""Store tier off the GPU: session rows in pinned host memory or on another GPU.

The reference keeps every stored row in the serving GPU's memory
(``src/marathon/shift_store.py:251-253``; ``docs/protocol.md:49`` lists no
other tier).  Here a :class:`~marathon_b200.shift_store.ShiftStore` built with
``device="cpu"`` holds its buffers in pinned host memory, and one built with
another GPU's device holds them there.  No kernel ever dereferences those
buffers: :class:`StagedMover` copies the rows a batch needs into a device
staging ring with the copy engines (``mshift_stage``: one ``cudaMemcpyAsync``
per contiguous range), and the ordinary batched kernels read the staging ring
as if it were a device store.  Saves run the other way: gather into staging,
then copy out.

Pipelining: the batch is cut into chunks (a group of whole layers when one
layer of the batch fits ``chunk_bytes``, else pieces of runs within one layer).
Chunk ``c`` is staged on a copy stream into slot ``c % 2`` while the kernel of
chunk ``c - 1`` runs on the compute stream; a slot is refilled only after the
kernel that read it has finished.  The transfer over the host link (or NVLink
for a peer GPU) is the bound; the kernels hide behind it.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .shift_kernels import Launcher, RunSpec, ShiftError, StoreView

#: default bytes of one staging slot (two slots are allocated)
DEFAULT_CHUNK_BYTES = 256 << 20

_ELEM_BYTES = {_lib.BF16: 2, _lib.F16: 2, _lib.F32: 4, _lib.E4M3: 1}


@dataclass
class Piece:
    """Tokens ``[offset, offset + length)`` of run ``run`` of the batch."""

    run: int
    offset: int
    length: int


@dataclass
class Chunk:
    """Layers ``[first_layer, +n_layers)`` x ``pieces``, staged as one slot.

    In the slot, layer ``i`` of the chunk starts at ``i * layer_bytes`` and
    piece ``j`` at ``offsets[j]`` within it; each piece's rows are dense.
    """

    first_layer: int
    n_layers: int
    pieces: list[Piece]
    offsets: list[int]
    layer_bytes: int

    @property
    def nbytes(self) -> int:
        return self.n_layers * self.layer_bytes


def plan_chunks(lengths: list[int], row_bytes: int, n_layers: int,
                chunk_bytes: int = DEFAULT_CHUNK_BYTES) -> list[Chunk]:
    """Cut ``runs x layers`` into staging chunks of at most ``chunk_bytes``.

    Every (run token, layer) lands in exactly one chunk.  Each chunk covers
    whole layers; when one layer of the batch is larger than a chunk, runs are
    split into pieces and each chunk covers one layer.  A chunk is never
    smaller than one row, so ``chunk_bytes`` below ``row_bytes`` still plans.
    """
    if row_bytes <= 0 or row_bytes % 16:
        raise ShiftError(f"store rows of {row_bytes} bytes: need a positive multiple of 16")
    if n_layers <= 0 or not lengths or min(lengths) <= 0:
        raise ShiftError("a staged batch needs layers and runs of positive length")
    chunk_bytes = max(int(chunk_bytes), row_bytes)
    per_layer = sum(lengths) * row_bytes
    if per_layer <= chunk_bytes:
        per = max(1, chunk_bytes // per_layer)
        pieces = [Piece(i, 0, n) for i, n in enumerate(lengths)]
        offsets = np.concatenate(([0], np.cumsum(lengths[:-1]))).astype(np.int64) * row_bytes
        # the first chunk is one layer: a consumer waiting for layer 0 waits
        # for one layer's transfer, not a whole chunk's
        starts = [0] + list(range(1, n_layers, per)) if per > 1 else list(range(n_layers))
        return [
            Chunk(l0, min(per if l0 else 1, n_layers - l0), pieces, offsets.tolist(), per_layer)
            for l0 in starts
        ]
    groups: list[list[Piece]] = []
    cur: list[Piece] = []
    room = chunk_bytes // row_bytes  # rows left in the current chunk
    for i, n in enumerate(lengths):
        off = 0
        while off < n:
            if room == 0:
                groups.append(cur)
                cur, room = [], chunk_bytes // row_bytes
            take = min(n - off, room)
            cur.append(Piece(i, off, take))
            off += take
            room -= take
    if cur:
        groups.append(cur)
    chunks = []
    for layer in range(n_layers):
        for g in groups:
            offs = np.concatenate(([0], np.cumsum([p.length for p in g][:-1]))) * row_bytes
            chunks.append(Chunk(layer, 1, g, offs.astype(np.int64).tolist(),
                                sum(p.length for p in g) * row_bytes))
    return chunks


def store_device(store_device_name: str) -> torch.device:
    d = torch.device(store_device_name)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


def is_staged(store_device_name: str, cache_device: torch.device) -> bool:
    """Whether a store on ``store_device_name`` must be staged for caches on ``cache_device``."""
    d = torch.device(store_device_name)
    if d.type == "cpu":
        return True
    if d.type != "cuda":
        raise ShiftError(f"a store on {d} is not supported")
    return d.index is not None and d.index != cache_device.index


@dataclass
class StagedLoad:
    """A staged load in flight: one completion event per cache layer.

    ``wait_layer(i)`` makes a stream wait until layer ``i``'s rows are in the
    paged cache (vLLM's ``wait_for_layer_load``); ``check()`` waits for the
    whole load on the host and raises on any rejected token.
    """

    layer_done: list
    last: torch.cuda.Event
    errs: torch.Tensor
    n_chunks: int
    #: queued on the caller's own stream (a device store): work queued there
    #: later is ordered after it without waiting on the host
    same_stream: bool = False

    def wait_layer(self, layer: int, stream=None) -> None:
        (stream or torch.cuda.current_stream()).wait_event(self.layer_done[layer])

    def wait_all(self, stream=None) -> None:
        (stream or torch.cuda.current_stream()).wait_event(self.last)

    def check(self) -> None:
        self.last.synchronize()
        bits = int(np.bitwise_or.reduce(self.errs[: self.n_chunks].numpy()))
        if bits:
            raise ShiftError(f"staged shift load: {_lib.describe_bits(bits)} (error bits {bits:#x})")


class StagedMover:
    """Batched load/save between an off-GPU store and the paged caches, through staging."""

    #: descriptor slots of the mover's own launcher: enough that issuing a whole
    #: load's chunks rarely waits on the host for an earlier chunk's kernel
    DESCRIPTOR_SLOTS = 64

    def __init__(self, launcher: Launcher, chunk_bytes: int = DEFAULT_CHUNK_BYTES) -> None:
        self.launcher = Launcher(launcher.layers, staging_slots=self.DESCRIPTOR_SLOTS)
        self.device = launcher.device
        self.lib = launcher.lib
        self.chunk_bytes = int(chunk_bytes)
        self.row_bytes_per_elem = _ELEM_BYTES[launcher.geo.dtype]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.load_stream = torch.cuda.Stream(self.device)  # kernels of asynchronous loads
        self._slots: list[torch.Tensor | None] = [None, None]
        self._freed: list[torch.cuda.Event | None] = [None, None]
        self._peers: set[int] = set()
        self.last_chunks = 0
        self.last_copies = 0
        self.last_staged_bytes = 0

    # ------------------------------------------------------------ helpers
    def enable_peer(self, peer: int) -> None:
        """Direct copies from GPU ``peer`` (a store tier there); once per peer."""
        if peer in self._peers or peer == self.device.index:
            return
        with torch.cuda.device(self.device):
            _lib.check(self.lib.mshift_enable_peer(int(peer)), "mshift_enable_peer")
        self._peers.add(peer)

    def _slot(self, k: int, nbytes: int) -> int:
        buf = self._slots[k]
        if buf is None or buf.numel() < nbytes:
            if self._freed[k] is not None:
                self._freed[k].synchronize()
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
            # used on the mover's own streams: the allocator must not hand the
            # memory out again while work queued there may still touch it
            buf.record_stream(self.copy_stream)
            buf.record_stream(self.load_stream)
            self._slots[k] = buf
        return buf.data_ptr()

    @staticmethod
    def _err_buffer(n: int) -> torch.Tensor:
        """Pinned error words of one call's chunks.  Fresh per call: the pinned-memory
        cache hands a block out again only after the copies into it completed."""
        return torch.zeros(n, dtype=torch.int32, pin_memory=True)

    @staticmethod
    def _check_runs(runs: list[RunSpec], store: StoreView, n_layers: int) -> None:
        """Host-side range checks: staged copies read host/peer memory directly."""
        S, L = store.ptrs.shape
        if L != n_layers:
            raise ShiftError(f"store view has {L} layers, the batch covers {n_layers}")
        for i, r in enumerate(runs):
            if not 0 <= r.session < S:
                raise ShiftError(f"run {i}: session row {r.session} of {S}")
            if r.length <= 0 or r.store_start < 0 or r.store_start + r.length > store.caps[r.session]:
                raise ShiftError(f"run {i}: store rows [{r.store_start}, +{r.length}) outside "
                                 f"capacity {store.caps[r.session]}")
            if not store.ptrs[r.session].all():
                raise ShiftError(f"run {i}: session row {r.session} lacks a layer buffer")

    @staticmethod
    def _copies(ch: Chunk, runs: list[RunSpec], store: StoreView, row_bytes: int,
                base: int, to_slot: bool) -> np.ndarray:
        """The chunk's ranges as ``mshift_copy`` records (store <-> slot)."""
        n_p = len(ch.pieces)
        rec = np.empty(ch.n_layers * n_p, dtype=_lib.COPY_DTYPE)
        sess = np.fromiter((runs[p.run].session for p in ch.pieces), np.int64, n_p)
        start = np.fromiter((runs[p.run].store_start + p.offset for p in ch.pieces), np.int64, n_p)
        nb = np.fromiter((p.length for p in ch.pieces), np.int64, n_p) * row_bytes
        offs = np.asarray(ch.offsets, dtype=np.int64)
        layers = np.arange(ch.first_layer, ch.first_layer + ch.n_layers)
        remote = (store.ptrs[sess[None, :], layers[:, None]].astype(np.int64)
                  + start[None, :] * row_bytes)
        local = base + np.arange(ch.n_layers, dtype=np.int64)[:, None] * ch.layer_bytes + offs[None, :]
        dst, src = (local, remote) if to_slot else (remote, local)
        rec["dst"] = dst.reshape(-1).astype(np.uint64)
        rec["src"] = src.reshape(-1).astype(np.uint64)
        rec["bytes"] = np.broadcast_to(nb[None, :], (ch.n_layers, n_p)).reshape(-1)
        return rec

    @staticmethod
    def _slot_view(ch: Chunk, base: int, store: StoreView) -> StoreView:
        """The slot as a device store: one session row per piece, rows from 0."""
        ptrs = (base + np.arange(ch.n_layers, dtype=np.int64)[None, :] * ch.layer_bytes
                + np.asarray(ch.offsets, dtype=np.int64)[:, None])
        caps = np.asarray([p.length for p in ch.pieces], dtype=np.int64)
        return StoreView(ptrs.astype(np.uint64), caps, store.st_tok, store.st_head)

    @staticmethod
    def _piece_runs(ch: Chunk, runs: list[RunSpec]) -> list[RunSpec]:
        out = []
        for j, p in enumerate(ch.pieces):
            r = runs[p.run]
            if r.slots is not None:
                out.append(RunSpec(j, 0, p.length, r.delta,
                                   slots=r.slots[p.offset : p.offset + p.length]))
            else:
                out.append(RunSpec(j, 0, p.length, r.delta, block_table=r.block_table,
                                   paged_start=r.paged_start + p.offset))
        return out

    def _stage(self, rec: np.ndarray, stream) -> None:
        _lib.check(self.lib.mshift_stage(rec.ctypes.data, len(rec), stream.cuda_stream),
                   "mshift_stage")

    def _row_bytes(self, store: StoreView) -> int:
        geo = self.launcher.geo
        if store.st_head != 2 * geo.head_size or store.st_tok != geo.heads * store.st_head:
            raise ShiftError("a staged store needs dense rows [heads, 2*head_size]")
        return int(store.st_tok) * self.row_bytes_per_elem

    # --------------------------------------------------------------- load
    def load(self, runs: list[RunSpec], store: StoreView, inv_freq: torch.Tensor, *,
             k_scales: torch.Tensor | None = None, check: bool = True) -> None:
        """Every run x every layer from the off-GPU store into the paged caches,
        ordered on the current stream."""
        if not runs:
            return
        job = self._load(runs, store, inv_freq, k_scales, torch.cuda.current_stream(self.device))
        if check:
            job.check()

    def load_async(self, runs: list[RunSpec], store: StoreView, inv_freq: torch.Tensor, *,
                   k_scales: torch.Tensor | None = None) -> StagedLoad | None:
        """The same load on the mover's own streams, returning at once.

        It starts after the work already queued on the current stream; layer
        ``i`` is in place once ``StagedLoad.wait_layer(i)``'s event fires, so a
        forward pass can run layer ``i`` while later layers are still crossing
        the host link.  Errors surface in ``StagedLoad.check()``.
        """
        if not runs:
            return None
        self.load_stream.wait_stream(torch.cuda.current_stream(self.device))
        return self._load(runs, store, inv_freq, k_scales, self.load_stream)

    def _load(self, runs, store, inv_freq, k_scales, compute) -> StagedLoad:
        n_layers = len(self.launcher.layers)
        self._check_runs(runs, store, n_layers)
        row_bytes = self._row_bytes(store)
        chunks = plan_chunks([r.length for r in runs], row_bytes, n_layers, self.chunk_bytes)
        size = max(c.nbytes for c in chunks)
        errs = self._err_buffer(len(chunks))
        layer_done: list = [None] * n_layers
        copies = 0
        # the copy stream must not overtake earlier work on the compute stream
        # (a save whose rows this load reads back, a cache the caller filled)
        self.copy_stream.wait_stream(compute)
        with torch.cuda.stream(compute):
            for ci, ch in enumerate(chunks):
                k = ci % 2
                base = self._slot(k, size)
                rec = self._copies(ch, runs, store, row_bytes, base, to_slot=True)
                # the chunk's descriptors ride the copy stream just ahead of its
                # rows: a descriptor copy queued on the compute stream would wait
                # in the copy engine behind the next chunk's rows
                view = self._slot_view(ch, base, store)
                p = self.launcher.prepare_load(self._piece_runs(ch, runs), view, inv_freq,
                                               k_scales=k_scales, first_layer=ch.first_layer,
                                               n_layers=ch.n_layers,
                                               upload_stream=self.copy_stream)
                if self._freed[k] is not None:
                    self.copy_stream.wait_event(self._freed[k])  # its last reader is done
                self._stage(rec, self.copy_stream)
                copies += len(rec)
                staged = torch.cuda.Event()
                staged.record(self.copy_stream)
                compute.wait_event(staged)
                self.launcher.launch(p)
                self.launcher.staging.copy_err(p.slot, errs[ci : ci + 1], compute)
                self.launcher.finish(p, False)
                freed = torch.cuda.Event()
                freed.record(compute)
                self._freed[k] = freed
                for layer in range(ch.first_layer, ch.first_layer + ch.n_layers):
                    layer_done[layer] = freed  # the layer's last chunk so far
        self.last_chunks, self.last_copies = len(chunks), copies
        self.last_staged_bytes = sum(c.nbytes for c in chunks)
        return StagedLoad(layer_done, freed, errs, len(chunks))

    # --------------------------------------------------------------- save
    def save(self, runs: list[RunSpec], store: StoreView, *, first_layer: int = 0,
             n_layers: int | None = None, check: bool = True, err: int | None = None) -> None:
        """Paged rows of every run x layers ``[first_layer, +n_layers)`` out to the store.

        ``err``: a device status word every chunk's kernel ORs its rejected-token
        bits into, read by the caller (with ``check=False``).
        """
        if not runs:
            return
        n_layers = self.launcher.layer_range(first_layer, n_layers)
        self._check_runs(runs, store, n_layers)
        row_bytes = self._row_bytes(store)
        chunks = plan_chunks([r.length for r in runs], row_bytes, n_layers, self.chunk_bytes)
        size = max(c.nbytes for c in chunks)
        compute = torch.cuda.current_stream(self.device)
        errs = self._err_buffer(len(chunks))
        copies = 0
        for ci, ch in enumerate(chunks):
            k = ci % 2
            base = self._slot(k, size)
            if self._freed[k] is not None:
                compute.wait_event(self._freed[k])  # the slot's last user is done
            view = self._slot_view(ch, base, store)
            p = self.launcher.prepare_save(self._piece_runs(ch, runs), view,
                                           first_layer=first_layer + ch.first_layer,
                                           n_layers=ch.n_layers)
            self.launcher.launch(p, err=err)
            if err is None:
                self.launcher.staging.copy_err(p.slot, errs[ci : ci + 1], compute)
            self.launcher.finish(p, False)
            gathered = torch.cuda.Event()
            gathered.record(compute)
            self.copy_stream.wait_event(gathered)
            rec = self._copies(ch, runs, store, row_bytes, base, to_slot=False)
            self._stage(rec, self.copy_stream)
            copies += len(rec)
            freed = torch.cuda.Event()
            freed.record(self.copy_stream)
            self._freed[k] = freed
        compute.wait_stream(self.copy_stream)  # later work on the stream sees the rows out
        self.last_chunks, self.last_copies = len(chunks), copies
        self.last_staged_bytes = sum(c.nbytes for c in chunks)
        if check and err is None:
            self._raise(compute, errs, len(chunks), "staged shift save")

    @staticmethod
    def _raise(stream, errs: torch.Tensor, n: int, what: str) -> None:
        stream.synchronize()
        bits = int(np.bitwise_or.reduce(errs[:n].numpy())) if n else 0
        if bits:
            raise ShiftError(f"{what}: {_lib.describe_bits(bits)} (error bits {bits:#x})")
