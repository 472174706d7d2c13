"""Re-rotate-and-scatter (load) and paged gather (save) on B200, behind the reference API.

Drop-in surface of the reference's ``marathon.shift_kernels``
(``src/marathon/shift_kernels.py``):

* :class:`RopeShift` / :func:`rope_shift` — per-delta rotation tables
  (``:50-84``).  The kernel reads one ``[2, rotary/2]`` fp32 table (cos, sin);
  the reference's ``cos``/``sgn``/``partner``/``emb_cos``/``emb_sin`` views
  are kept on the object for callers that use them.
* :func:`scatter_shifted` — one layer, one run (``:166-210``).
* :func:`warmup` — the reference pre-compiled Triton here (``:213-238``); the
  sm_100a kernels are compiled ahead of time, so this only loads the library
  and resolves the launch grid.

plus the batched entry points the connector uses, :class:`Launcher.load` and
:class:`Launcher.save`, which run every run x every layer x every session of a
step in one persistent launch each.

There is no CPU path: a CPU tensor, a missing library or a non-zero native
status raises :class:`ShiftError`.
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import RUN_DTYPE, ShiftError
from .paged import KVLayers, PagedLayout, describe, paged_strides

__all__ = [
    "RopeShift",
    "rope_shift",
    "rope_tables",
    "scatter_shifted",
    "set_load_kernel",
    "warmup",
    "inv_freq",
    "RunSpec",
    "StoreView",
    "Launcher",
    "ShiftError",
    "paged_strides",
]


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ShiftError(
            f"{what} is on {t.device}: the shift kernels are CUDA-only and have no CPU path"
        )


def inv_freq(rotary: int, theta: float) -> torch.Tensor:
    """RoPE inverse frequencies exactly as the connector forms them (fp32, on CPU).

    ``1 / theta ** (arange(0, rotary, 2) / rotary)``
    (``src/marathon/vllm_shift_connector.py:196-198``).
    """
    return 1.0 / (theta ** (torch.arange(0, rotary, 2, dtype=torch.float32) / rotary))


# ------------------------------------------------------------------ tables
@dataclass(frozen=True)
class RopeShift:
    """Rotation tables of one delta on the device the kernel runs on.

    ``table`` (``[2, rotary/2]``: cos then sin of ``fp32(delta) * inv_freq``) is
    what the kernel reads.  ``cos``/``sgn``/``partner``/``emb_cos``/``emb_sin``
    are the reference's branchless and broadcast forms of the same numbers
    (``src/marathon/shift_kernels.py:50-65``): ``out[i] = k[i]*cos[i] +
    k[partner[i]]*sgn[i]``, with a non-rotary tail of ``cos = 1, sgn = 0``.
    """

    delta: int
    cos: torch.Tensor
    sgn: torch.Tensor
    partner: torch.Tensor
    emb_cos: torch.Tensor
    emb_sin: torch.Tensor
    table: torch.Tensor = field(repr=False)

    @property
    def rotary(self) -> int:
        return int(self.emb_cos.numel())


def rope_tables(deltas: torch.Tensor, inv: torch.Tensor) -> torch.Tensor:
    """``[n, 2, half]`` cos/sin tables for ``n`` deltas in one launch (device tensors)."""
    _require_cuda(deltas, "deltas")
    _require_cuda(inv, "inv_freq")
    deltas = deltas.to(torch.int64).contiguous()
    inv = inv.to(torch.float32).contiguous()
    half = int(inv.numel())
    out = torch.empty((deltas.numel(), 2, half), dtype=torch.float32, device=deltas.device)
    lib = _lib.load()
    _lib.check(
        lib.mshift_rope_tables(
            deltas.data_ptr(), deltas.numel(), inv.data_ptr(), half, out.data_ptr(),
            _stream_ptr(deltas.device),
        ),
        "mshift_rope_tables",
    )
    return out


def rope_shift(delta: int, head_size: int, inv_freq: torch.Tensor, device) -> RopeShift:
    """Tables that move RoPE'd keys ``delta`` positions, for one head dimension.

    Same signature and fields as the reference (``shift_kernels.py:68-84``);
    the numbers come from the native table kernel.
    """
    device = torch.device(device)
    if device.type != "cuda":
        raise ShiftError("rope_shift builds its tables with a CUDA kernel; pass a CUDA device")
    rotary = 2 * int(inv_freq.numel())
    if rotary > head_size:
        raise ShiftError(f"rotary {rotary} > head_size {head_size}")
    half = rotary // 2
    inv = inv_freq.to(device=device, dtype=torch.float32)
    table = rope_tables(torch.tensor([int(delta)], dtype=torch.int64, device=device), inv)[0]
    c, s = table[0], table[1]
    cos = torch.ones(head_size, dtype=torch.float32, device=device)
    sgn = torch.zeros(head_size, dtype=torch.float32, device=device)
    cos[:rotary] = torch.cat((c, c))
    sgn[:half] = -s
    sgn[half:rotary] = s
    partner = torch.arange(head_size, dtype=torch.int32, device=device)
    partner[:half] += half
    partner[half:rotary] -= half
    return RopeShift(int(delta), cos, sgn, partner, torch.cat((c, c)), torch.cat((s, s)), table)


def set_load_kernel(kind: str) -> str:
    """Select the load kernel process-wide: ``"auto"`` (default), ``"lsu"`` or ``"bulk"``.

    Returns the previous selection.  All write identical bits; they differ in
    how the store rows reach the SM (128-bit loads vs one TMA bulk copy per
    stage).  ``"auto"`` uses TMA for e4m3 caches and 128-bit loads otherwise.
    """
    codes = {"lsu": _lib.KERNEL_LSU, "bulk": _lib.KERNEL_BULK, "auto": _lib.KERNEL_AUTO}
    if kind not in codes:
        raise ShiftError(f"unknown load kernel {kind!r}")
    prev = _lib.load().mshift_set_load_kernel(codes[kind])
    return {v: k for k, v in codes.items()}[prev]


# ------------------------------------------------------------ error words
_ERR: dict[int, torch.Tensor] = {}


def _err_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=device)
        _ERR[idx] = t
    return t


def take_errors(device=None) -> int:
    """Synchronise, return and clear the error bits accumulated by unchecked launches."""
    device = torch.device(device if device is not None else "cuda")
    t = _err_word(device)
    bits = int(t[0].item())
    t.zero_()
    return bits


def _raise_bits(bits: int, what: str) -> None:
    if bits:
        raise ShiftError(f"{what}: kernel rejected tokens ({_lib.describe_bits(bits)}); "
                         "those tokens were not written")


# ------------------------------------------------------------ single layer
def scatter_shifted(
    src: torch.Tensor,
    kv: torch.Tensor,
    slots: torch.Tensor,
    block_size: int,
    hnd: bool,
    shift: RopeShift | None,
    *,
    k_scale: torch.Tensor | None = None,
    fp8: bool = False,
    check: bool = False,
) -> None:
    """Write ``src`` (``[n, heads, 2*head_size]``) into ``kv``'s slots, K rotated by delta.

    Contract of the reference (``shift_kernels.py:166-210``): ``slots`` are
    flat destination slots (block ``slot // block_size``, offset
    ``slot % block_size``), ``hnd`` selects the fused layout, ``shift=None`` or
    delta 0 is a plain scatter, ``n == 0`` is a no-op.  ``src`` must have the
    cache's dtype (the store holds cache-dtype rows).  E4M3 caches
    (``float8_e4m3fn``, or ``uint8`` with ``fp8=True``) are dequantised,
    rotated and requantised with the layer's K scale, which cancels: the
    kernel rotates the codes' values and rounds once, so ``k_scale`` is
    accepted for the reference's call shape but not needed.  ``check=True`` synchronises and raises on
    any token the kernel rejected; otherwise rejections accumulate for
    :func:`take_errors`.
    """
    _require_cuda(kv, "kv")
    n, heads, two_d = src.shape
    if kv.shape[-1] != two_d:
        raise ShiftError(f"src row {two_d} != kv row {kv.shape[-1]}")
    if n == 0:
        return
    _require_cuda(src, "src")
    _require_cuda(slots, "slots")
    if src.dtype != kv.dtype:
        raise ShiftError(f"src dtype {src.dtype} != cache dtype {kv.dtype}")
    if src.stride(-1) != 1:
        raise ShiftError("src rows must be contiguous in the head dimension")
    geo = describe(kv, block_size, "hnd" if hnd else "nhd", fp8=fp8)
    if geo.heads != heads:
        raise ShiftError(f"src has {heads} heads, cache has {geo.heads}")
    slots = slots.to(torch.int64).contiguous()
    if slots.numel() != n:
        raise ShiftError(f"{slots.numel()} slots for {n} tokens")
    rotate = shift is not None and shift.delta != 0
    rotary = shift.rotary if shift is not None else geo.head_size
    table_ptr = shift.table.data_ptr() if rotate else None
    ks_ptr = None  # e4m3: the K scale cancels; the kernel does not read it
    err = _err_word(kv.device)
    k_base = kv.data_ptr()
    v_base = k_base + geo.head_size * geo.elem_bytes
    lib = _lib.load()
    paged = geo.struct()
    _lib.check(
        lib.mshift_scatter_shifted(
            src.data_ptr(), src.stride(0), src.stride(1), n, k_base, v_base,
            ctypes.byref(paged), slots.data_ptr(), table_ptr, rotary, ks_ptr,
            err.data_ptr(), _stream_ptr(kv.device),
        ),
        "mshift_scatter_shifted",
    )
    if check:
        _raise_bits(take_errors(kv.device), "scatter_shifted")


def warmup(kv: torch.Tensor, block_size: int, hnd: bool, *, rotary: int | None = None,
           layout: str | None = None, fp8: bool = False) -> None:
    """Load the library and validate ``kv``'s geometry before the first real load.

    The reference JIT-compiled Triton here (``shift_kernels.py:213-238``) and
    its connector called it from ``register_kv_caches``
    (``vllm_shift_connector.py:405``), so a geometry no kernel serves failed at
    registration rather than at the first load.  The native kernels are
    compiled ahead of time: this loads the library and raises
    :class:`ShiftError` when no compiled kernel serves ``kv``'s dtype, head
    size and ``rotary`` (default: the whole head).  ``layout`` (``"nhd"``,
    ``"hnd"``, ``"split"``, ``"split_blocks"``) overrides ``hnd`` for the 5-D
    split caches; ``fp8`` marks a ``uint8`` cache as e4m3 codes.
    """
    lib = _lib.load()
    if not kv.is_cuda:
        return
    geo = describe(kv, block_size, layout or ("hnd" if hnd else "nhd"), fp8=fp8)
    rot = geo.head_size if rotary is None else int(rotary)
    if not lib.mshift_supported(geo.dtype, geo.head_size, rot):
        raise ShiftError(f"no kernel for dtype code {geo.dtype}, head_size {geo.head_size}, "
                         f"rotary {rot}")


# ------------------------------------------------------------------ batches
@dataclass(slots=True)
class RunSpec:
    """One run of a batch: ``length`` tokens of ``session`` starting at ``store_start``.

    The paged side is ``slots`` (CUDA int64 ``[length]``, the reference's
    ``_Load.slots``) or ``block_table`` plus ``paged_start`` (the logical
    position of the first token).  A ``block_table`` given as a host sequence
    or numpy array travels to the device inside the batch's single descriptor
    copy; a CUDA int32 tensor is used in place.  ``delta`` is the RoPE offset
    of a load (ignored by saves).
    """

    session: int
    store_start: int
    length: int
    delta: int = 0
    slots: torch.Tensor | None = None
    block_table: object = None
    paged_start: int = 0


@dataclass
class StoreView:
    """Store buffers of the sessions in a batch, indexed [session row][layer]."""

    ptrs: np.ndarray  # uint64 [n_sessions, n_layers]; 0 = missing buffer
    caps: np.ndarray  # int64 [n_sessions]
    st_tok: int
    st_head: int
    keepalive: list = field(default_factory=list, repr=False)

    def __post_init__(self) -> None:
        self.ptrs = np.ascontiguousarray(self.ptrs, dtype=np.uint64)
        self.caps = np.ascontiguousarray(self.caps, dtype=np.int64)


def _align(n: int, a: int = 16) -> int:
    return (n + a - 1) // a * a


class _Staging:
    """Pinned host + device staging of one batch's descriptors, a ring of slots.

    A batch's descriptors — run records, store pointer table, capacities,
    deltas, host block tables and a zeroed error word — reach the device in
    ONE host-to-device copy.  Slots rotate (four by default for a launcher) so
    the host can pack batches while earlier batches' kernels still read theirs,
    up to that many batches ahead of the GPU.  The copies
    go through ``mshift_stage`` (one ``cudaMemcpyAsync`` each) with records
    prepared once per slot.
    """

    def __init__(self, device: torch.device, lib, slots: int = 2) -> None:
        self.device = device
        self.lib = lib
        self.n = int(slots)
        self.cap = 0
        self.host: list[torch.Tensor] = []
        self.dev: list[torch.Tensor] = []
        self.done = [torch.cuda.Event() for _ in range(self.n)]
        self.used = [False] * self.n
        self.slot = 0
        self.err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._status_stream = None  # status-word read-backs off the launch stream
        # per slot: [upload record, error-word read-back record]
        self.rec = np.zeros((self.n, 2), dtype=_lib.COPY_DTYPE)
        self.rec_addr = self.rec.ctypes.data

    def _ensure(self, n: int) -> None:
        if n <= self.cap:
            return
        for k in range(self.n):
            if self.used[k]:
                self.done[k].synchronize()
        cap = 1 << max(12, (n - 1).bit_length())
        self.host = [torch.empty(cap, dtype=torch.uint8).pin_memory() for _ in range(self.n)]
        self.host_np = [h.numpy() for h in self.host]
        self.dev = [torch.empty(cap, dtype=torch.uint8, device=self.device) for _ in range(self.n)]
        self.dev_ptr = [d.data_ptr() for d in self.dev]
        for k in range(self.n):
            self.rec[k, 0] = (self.dev_ptr[k], self.host[k].data_ptr(), 0)
            self.rec[k, 1] = (self.err_host.data_ptr(), self.dev_ptr[k], 4)
        self.cap = cap

    def begin(self, n: int) -> tuple[int, np.ndarray, int]:
        """Pick the next slot, waiting for its previous batch: (slot, host view, device base)."""
        self._ensure(n)
        slot = self.slot
        self.slot = (slot + 1) % self.n
        if self.used[slot]:
            self.done[slot].synchronize()
        return slot, self.host_np[slot], self.dev_ptr[slot]

    def upload(self, slot: int, n: int, stream_ptr: int) -> None:
        self.rec[slot, 0]["bytes"] = n
        _lib.check(self.lib.mshift_stage(self.rec_addr + slot * 2 * _lib.COPY_DTYPE.itemsize, 1,
                                         stream_ptr), "mshift_stage (descriptors)")

    def finish(self, slot: int, stream) -> None:
        """The slot's latest use is queued on ``stream``: ``begin`` waits for it."""
        self.done[slot].record(stream)
        self.used[slot] = True

    def drain(self) -> None:
        for k in range(self.n):
            if self.used[k]:
                self.done[k].synchronize()

    def copy_err(self, slot: int, dst: torch.Tensor, stream) -> None:
        """Queue a copy of the slot's error word into ``dst`` (pinned int32 [1]) on ``stream``."""
        with torch.cuda.stream(stream):
            dst.copy_(self.dev[slot][:4].view(torch.int32), non_blocking=True)

    def copy_err_after(self, slot: int, dst: torch.Tensor, after) -> torch.cuda.Event:
        """Copy the slot's error word into ``dst`` (pinned int32 [1]) once the event
        ``after`` (recorded behind the batch's kernels) has completed, on a side
        stream of the ring's own; returns the event that marks the copy done.

        Nothing is queued on the launch stream: a copy there would sit between
        this batch's load kernel and the next batch's table kernel, which then
        could no longer launch while the load finishes (programmatic dependent
        launch).  The slot stays busy until the copy has read the word, so the
        next batch's descriptor upload cannot zero it first.
        """
        if self._status_stream is None:
            self._status_stream = torch.cuda.Stream(self.device)
        st = self._status_stream
        st.wait_event(after)
        with torch.cuda.stream(st):
            dst.copy_(self.dev[slot][:4].view(torch.int32), non_blocking=True)
        done = torch.cuda.Event()
        done.record(st)
        self.finish(slot, st)
        return done

    def read_err(self, slot: int, stream) -> int:
        rec = self.rec_addr + (slot * 2 + 1) * _lib.COPY_DTYPE.itemsize
        _lib.check(self.lib.mshift_stage(rec, 1, stream.cuda_stream), "mshift_stage (status)")
        stream.synchronize()
        return int(self.err_host[0])


@dataclass
class Prepared:
    """A staged batch: descriptors on the device, ready to launch."""

    kind: str  # "load" | "save"
    slot: int
    base: int  # device address of the staging slot (error word at +0)
    runs: int
    n_runs: int
    tiles: int
    n_layers: int
    first_layer: int
    ptrs: int
    caps: int
    n_sessions: int
    st_tok: int
    st_head: int
    deltas: int
    n_deltas: int
    h2d_bytes: int
    tile_tokens: int = 0
    tables: torch.Tensor | None = None
    k_scales: torch.Tensor | None = None
    inv_freq: torch.Tensor | None = None
    stream: object = None  # the torch stream current when the batch was prepared
    uploaded: object = None  # event after the descriptor copy, when it ran on the copy stream


class Launcher:
    """Batched load/save over registered paged caches, one persistent launch per call.

    ``layers`` is the :class:`KVLayers` of this rank's caches.  ``load`` /
    ``save`` = :meth:`prepare_load` / :meth:`prepare_save` (pack on the host,
    one H2D copy) + :meth:`launch` (native calls only) + an optional error
    check (one 4-byte D2H read and a stream sync).
    """

    def __init__(self, layers: KVLayers, tile_tokens: int | None = None,
                 staging_slots: int = 4) -> None:
        if layers.k_ptrs is None:
            raise ShiftError("the batched kernels need CUDA caches")
        self.layers = layers
        self.geo: PagedLayout = layers.geometry
        self.device = layers.device
        self.lib = _lib.load()
        self.fixed_tile = tile_tokens is not None and tile_tokens > 0
        self.tile_tokens = int(tile_tokens or self.lib.mshift_default_tile_tokens(self.geo.heads))
        self.paged = self.geo.struct()
        props = torch.cuda.get_device_properties(self.device)
        self._grid = props.multi_processor_count * self.CTAS_PER_SM
        self.staging = _Staging(self.device, self.lib, staging_slots)
        self._copy_stream = None
        self._upload_events = [torch.cuda.Event() for _ in range(staging_slots)]
        self.last_launches = 0
        self.last_h2d = 0  # bytes of the last batch's descriptor copy
        self._tables: list[torch.Tensor | None] = [None] * staging_slots

    #: resident CTAs of the load/save kernel per SM (register-limited, B200)
    CTAS_PER_SM = 2

    #: copy a batch's descriptors on the launcher's own copy stream as soon as
    #: they are packed: the copy then overlaps whatever the launch stream is
    #: still running (the previous batch's kernels), and the launch stream waits
    #: on an event instead of serialising the copy in front of the kernels
    EARLY_UPLOAD = True

    def _upload(self, slot: int, total: int, stream, upload_stream):
        """Queue the slot's descriptor copy; returns the event a launch must wait on
        (None when the copy is on the launch stream itself).

        The slot counts as in use from here on, not only once its batch has
        launched: a batch prepared and then abandoned still has a copy in flight
        from the slot's pinned buffer, which the next ``begin`` of the slot
        must wait for.
        """
        if upload_stream is not None or not self.EARLY_UPLOAD:
            on = upload_stream or stream
            self.staging.upload(slot, total, on.cuda_stream)
            self.staging.finish(slot, on)
            return None
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.device)
        # the slot's previous batch has finished (begin() waited for it), so
        # the copy may run ahead of the launch stream
        self.staging.upload(slot, total, self._copy_stream.cuda_stream)
        ev = self._upload_events[slot]
        ev.record(self._copy_stream)
        self.staging.finish(slot, self._copy_stream)
        return ev

    def drain(self) -> None:
        """Wait for every batch (and descriptor copy) issued from the staging slots.

        Call before dropping a launcher: its pinned slots are read by raw
        ``cudaMemcpyAsync`` calls the caching host allocator does not track.
        """
        self.staging.drain()

    #: (token, head) units per tile of a batched launch.  Both load kernels and
    #: the save kernel claim tiles dynamically, so a launch ends within one tile
    #: of its fastest CTA whatever the tile count; the tile only has to amortise
    #: its fixed cost (the claim, two barriers, slot resolution, table staging)
    #: and fill whole passes of 64 units.  Measured on B200 (c2 turn at 1/2/4/8
    #: heads per rank, tiles of 128-1024 units): 256 units is best or within
    #: noise of it up to about 64 tiles per resident CTA; beyond that (a full
    #: 8-head c2 turn has 121) 448 units is 0.7% faster.  An e4m3 cache is
    #: served by the TMA kernel, which splits a tile into 24 KiB stages: 384
    #: units (256 bytes each) are four full stages at any head count, and a
    #: ragged last stage costs about 3% (c3 turn, tiles of 192-1152 units).
    TILE_UNITS = 256
    TILE_UNITS_LARGE = 448
    TILE_UNITS_E4M3 = 384
    LARGE_TILES_PER_CTA = 64
    #: bounds of tokens per tile (the kernels accept 1..512)
    TILE_TOKENS_MIN, TILE_TOKENS_MAX = 16, 512

    def _tile_for(self, tokens: int, n_layers: int, lengths=None) -> int:
        """Tokens per tile for a batch of ``tokens`` tokens over ``n_layers`` layers.

        ``TILE_UNITS`` units per tile, or ``TILE_UNITS_LARGE`` for launches with
        more than ``LARGE_TILES_PER_CTA`` tiles of ``TILE_UNITS`` per resident
        CTA, or ``TILE_UNITS_E4M3`` for an e4m3 cache, divided by this rank's
        heads.
        """
        heads = self.geo.heads
        units = self.TILE_UNITS
        if self.geo.dtype == _lib.E4M3:
            units = self.TILE_UNITS_E4M3
        elif tokens * n_layers * heads > self.LARGE_TILES_PER_CTA * self._grid * self.TILE_UNITS:
            units = self.TILE_UNITS_LARGE
        return int(min(max(units // heads, self.TILE_TOKENS_MIN), self.TILE_TOKENS_MAX))

    # -- packing ------------------------------------------------------------
    _RUN = struct.Struct("<qqQQiiiiii")  # mshift_run, 56 bytes
    _SMALL = 32  # batches up to this many runs are packed record by record

    def _prepare(self, kind, runs, store, deltas, first_layer, n_layers, stream,
                 upload_stream=None) -> Prepared:
        if len(runs) <= self._SMALL:
            return self._prepare_small(kind, runs, store, deltas, first_layer, n_layers, stream,
                                       upload_stream)
        n_runs = len(runs)
        S, L = store.ptrs.shape
        if L != n_layers:
            raise ShiftError(f"store view has {L} layers, the launch covers {n_layers}")
        length = np.fromiter((r.length for r in runs), dtype=np.int64, count=n_runs)
        session = np.fromiter((r.session for r in runs), dtype=np.int64, count=n_runs)
        if n_runs and (length.min() <= 0 or session.min() < 0 or session.max() >= S):
            bad = int(np.argmax((length <= 0) | (session < 0) | (session >= S)))
            raise ShiftError(f"run {bad}: length {length[bad]}, session row {session[bad]} of {S}")
        tt = self.tile_tokens if self.fixed_tile else self._tile_for(
            int(length.sum()), n_layers, length.tolist() if n_runs <= 512 else None)
        self.tile_tokens = tt
        ntiles = (length + tt - 1) // tt
        tile_begin = np.zeros(n_runs, dtype=np.int64)
        if n_runs > 1:
            np.cumsum(ntiles[:-1], out=tile_begin[1:])
        tiles = int(ntiles.sum())
        if tiles * n_layers > 2**31 - 1:
            raise ShiftError("batch too large for one launch")

        # host block tables travel inside the staging copy, once per distinct table
        host_tables: dict[int, np.ndarray] = {}
        for r in runs:
            bt = r.block_table
            if r.slots is None and bt is not None and not isinstance(bt, torch.Tensor):
                if id(bt) not in host_tables:
                    host_tables[id(bt)] = np.ascontiguousarray(bt, dtype=np.int32)
        o_runs = 16
        o_ptrs = _align(o_runs + RUN_DTYPE.itemsize * n_runs)
        o_caps = _align(o_ptrs + 8 * S * L)
        o_deltas = _align(o_caps + 8 * S)
        tab_at, at = {}, _align(o_deltas + 8 * max(len(deltas), 1))
        for key, bt in host_tables.items():
            tab_at[key] = at
            at = _align(at + bt.nbytes)
        total = at

        slot, host, base = self.staging.begin(total)
        rec = np.zeros(n_runs, dtype=RUN_DTYPE)
        rec["store_start"] = np.fromiter((r.store_start for r in runs), dtype=np.int64,
                                         count=n_runs)
        rec["len"] = length
        rec["session"] = session
        rec["tile_begin"] = tile_begin
        table_of = {d: i for i, d in enumerate(deltas)}
        rec["table"] = [table_of.get(int(r.delta), -1) for r in runs]
        # per-run pointers gathered in lists, then written column by column
        # (element-wise writes into a structured array cost microseconds each)
        slots_col = [0] * n_runs
        bt_col = [0] * n_runs
        bt_len_col = [0] * n_runs
        start_col = [0] * n_runs
        for i, r in enumerate(runs):
            if r.slots is not None:
                if r.slots.dtype != torch.int64 or not r.slots.is_cuda or r.slots.numel() < r.length:
                    raise ShiftError(f"run {i}: slots must be a CUDA int64 tensor of >= {r.length}")
                slots_col[i] = r.slots.data_ptr()
                continue
            bt = r.block_table
            if bt is None:
                raise ShiftError(f"run {i} has neither slots nor a block table")
            if isinstance(bt, torch.Tensor):
                if bt.dtype != torch.int32 or not bt.is_cuda:
                    raise ShiftError(f"run {i}: a tensor block_table must be CUDA int32")
                bt_col[i] = bt.data_ptr()
                bt_len_col[i] = bt.numel()
            else:
                bt_col[i] = base + tab_at[id(bt)]
                bt_len_col[i] = host_tables[id(bt)].size
            start_col[i] = r.paged_start
        rec["slots"] = slots_col
        rec["block_table"] = bt_col
        rec["block_table_len"] = bt_len_col
        rec["paged_start"] = start_col

        host[:16] = 0  # the error word
        host[o_runs : o_runs + rec.nbytes] = rec.view(np.uint8)
        host[o_ptrs : o_ptrs + 8 * S * L] = (
            np.ascontiguousarray(store.ptrs, dtype=np.uint64).view(np.uint8).reshape(-1)
        )
        host[o_caps : o_caps + 8 * S] = np.ascontiguousarray(store.caps, dtype=np.int64).view(
            np.uint8
        )
        if deltas:
            host[o_deltas : o_deltas + 8 * len(deltas)] = np.asarray(deltas, dtype=np.int64).view(
                np.uint8
            )
        for key, bt in host_tables.items():
            host[tab_at[key] : tab_at[key] + bt.nbytes] = bt.view(np.uint8)
        uploaded = self._upload(slot, total, stream, upload_stream)
        self.last_h2d = total
        return Prepared(kind, slot, base, base + o_runs, n_runs, tiles, n_layers, first_layer,
                        base + o_ptrs, base + o_caps, S, store.st_tok, store.st_head,
                        base + o_deltas, len(deltas), total, tt, stream=stream,
                        uploaded=uploaded)

    def _prepare_small(self, kind, runs, store, deltas, first_layer, n_layers, stream,
                       upload_stream=None) -> Prepared:
        """``_prepare`` for a few runs: records packed straight into the pinned slot."""
        n_runs = len(runs)
        S, L = store.ptrs.shape
        if L != n_layers:
            raise ShiftError(f"store view has {L} layers, the launch covers {n_layers}")
        total_tokens = 0
        for i, r in enumerate(runs):
            if r.length <= 0 or not 0 <= r.session < S:
                raise ShiftError(f"run {i}: length {r.length}, session row {r.session} of {S}")
            total_tokens += r.length
        tt = self.tile_tokens if self.fixed_tile else self._tile_for(
            total_tokens, n_layers, [r.length for r in runs])
        self.tile_tokens = tt
        host_tables: dict[int, np.ndarray] = {}
        for r in runs:
            bt = r.block_table
            if r.slots is None and bt is not None and not isinstance(bt, torch.Tensor):
                if id(bt) not in host_tables:
                    host_tables[id(bt)] = np.ascontiguousarray(bt, dtype=np.int32)
        o_runs = 16
        o_ptrs = _align(o_runs + 56 * n_runs)
        o_caps = _align(o_ptrs + 8 * S * L)
        o_deltas = _align(o_caps + 8 * S)
        tab_at, at = {}, _align(o_deltas + 8 * max(len(deltas), 1))
        for key, bt in host_tables.items():
            tab_at[key] = at
            at = _align(at + bt.nbytes)
        total = at
        slot, host, base = self.staging.begin(total)
        table_of = {d: i for i, d in enumerate(deltas)}
        pack = self._RUN.pack_into
        tiles = 0
        for i, r in enumerate(runs):
            slots_ptr = bt_ptr = 0
            bt_len = 0
            paged_start = 0
            if r.slots is not None:
                if r.slots.dtype != torch.int64 or not r.slots.is_cuda or r.slots.numel() < r.length:
                    raise ShiftError(f"run {i}: slots must be a CUDA int64 tensor of >= {r.length}")
                slots_ptr = r.slots.data_ptr()
            else:
                bt = r.block_table
                if bt is None:
                    raise ShiftError(f"run {i} has neither slots nor a block table")
                if isinstance(bt, torch.Tensor):
                    if bt.dtype != torch.int32 or not bt.is_cuda:
                        raise ShiftError(f"run {i}: a tensor block_table must be CUDA int32")
                    bt_ptr, bt_len = bt.data_ptr(), bt.numel()
                else:
                    bt_ptr, bt_len = base + tab_at[id(bt)], host_tables[id(bt)].size
                paged_start = r.paged_start
            pack(host, o_runs + 56 * i, r.store_start, paged_start, slots_ptr, bt_ptr, bt_len,
                 r.length, r.session, table_of.get(int(r.delta), -1), tiles, 0)
            tiles += -(-r.length // tt)
        if tiles * n_layers > 2**31 - 1:
            raise ShiftError("batch too large for one launch")
        host[:16] = 0  # the error word
        host[o_ptrs : o_ptrs + 8 * S * L] = store.ptrs.view(np.uint8).reshape(-1)
        host[o_caps : o_caps + 8 * S] = store.caps.view(np.uint8)
        for k, d in enumerate(deltas):
            struct.pack_into("<q", host, o_deltas + 8 * k, d)
        for key, bt in host_tables.items():
            host[tab_at[key] : tab_at[key] + bt.nbytes] = bt.view(np.uint8)
        uploaded = self._upload(slot, total, stream, upload_stream)
        self.last_h2d = total
        return Prepared(kind, slot, base, base + o_runs, n_runs, tiles, n_layers, first_layer,
                        base + o_ptrs, base + o_caps, S, store.st_tok, store.st_head,
                        base + o_deltas, len(deltas), total, tt, stream=stream,
                        uploaded=uploaded)

    def prepare_load(
        self,
        runs: list[RunSpec],
        store: StoreView,
        inv_freq: torch.Tensor,
        *,
        k_scales: torch.Tensor | None = None,
        first_layer: int = 0,
        n_layers: int | None = None,
        upload_stream=None,
    ) -> Prepared:
        """Pack a load batch and queue its descriptor copy.

        The copy goes on the current stream, or on ``upload_stream`` when the
        caller orders it itself (it must complete before the batch's launch).
        """
        _require_cuda(inv_freq, "inv_freq")
        n_layers = self.layer_range(first_layer, n_layers)
        deltas = sorted({int(r.delta) for r in runs if int(r.delta) != 0})
        p = self._prepare("load", runs, store, deltas, first_layer, n_layers,
                          torch.cuda.current_stream(self.device), upload_stream)
        p.inv_freq = inv_freq if inv_freq.dtype == torch.float32 else inv_freq.float()
        # e4m3: the per-layer K scale cancels between dequantisation and
        # requantisation, so the kernels never read k_scales
        p.k_scales = None
        if deltas:
            # per staging slot, so a batch still in flight keeps its tables
            need = len(deltas) * 2 * p.inv_freq.numel()
            buf = self._tables[p.slot]
            if buf is None or buf.numel() < need:
                buf = torch.empty(max(need, 1024), dtype=torch.float32, device=self.device)
                self._tables[p.slot] = buf
            p.tables = buf
        return p

    def prepare_save(
        self, runs: list[RunSpec], store: StoreView, *, first_layer: int = 0,
        n_layers: int | None = None,
    ) -> Prepared:
        n_layers = self.layer_range(first_layer, n_layers)
        return self._prepare("save", runs, store, [], first_layer, n_layers,
                             torch.cuda.current_stream(self.device))

    def layer_range(self, first_layer: int, n_layers: int | None) -> int:
        """Layers of a batch starting at ``first_layer`` (default: to the last); raises
        if the range leaves the registered caches."""
        n_layers = len(self.layers) - first_layer if n_layers is None else int(n_layers)
        if first_layer < 0 or n_layers <= 0 or first_layer + n_layers > len(self.layers):
            raise ShiftError(f"layer range [{first_layer}, +{n_layers}) outside the caches")
        return n_layers

    def launch(self, p: Prepared, *, tables: bool = True, main: bool = True,
               err: int | None = None) -> int:
        """Issue the native launches of a prepared batch; returns how many were issued.

        The kernel ORs its rejected-token bits into the staging slot's status
        word, or into the device word at address ``err`` when given (a word
        the caller shares between several launches and reads once).
        """
        # a descriptor copy that has already completed needs no stream wait;
        # leaving it out keeps this batch's kernels directly behind the
        # previous batch's in the stream (programmatic dependent launch)
        if p.uploaded is not None and not p.uploaded.query():
            p.stream.wait_event(p.uploaded)
        stream = p.stream.cuda_stream
        err_ptr = p.base if err is None else int(err)
        n = 0
        if p.kind == "load":
            half = int(p.inv_freq.numel())
            if tables and p.n_deltas:
                _lib.check(
                    self.lib.mshift_rope_tables(p.deltas, p.n_deltas, p.inv_freq.data_ptr(), half,
                                                p.tables.data_ptr(), stream),
                    "mshift_rope_tables",
                )
                n += 1
            if main:
                off = 8 * p.first_layer
                _lib.check(
                    self.lib.mshift_load(
                        ctypes.byref(self.paged), 2 * half, p.runs, p.n_runs, p.tile_tokens,
                        p.tiles, p.n_layers, p.ptrs, p.caps, p.n_sessions, p.st_tok, p.st_head,
                        self.layers.k_ptrs.data_ptr() + off, self.layers.v_ptrs.data_ptr() + off,
                        p.tables.data_ptr() if p.tables is not None else None, p.n_deltas,
                        p.k_scales.data_ptr() + 4 * p.first_layer
                        if p.k_scales is not None else None,
                        err_ptr, stream,
                    ),
                    "mshift_load",
                )
                n += 1
        else:
            if main:
                off = 8 * p.first_layer
                _lib.check(
                    self.lib.mshift_save(
                        ctypes.byref(self.paged), p.runs, p.n_runs, p.tile_tokens, p.tiles,
                        p.n_layers, p.ptrs, p.caps, p.n_sessions, p.st_tok, p.st_head,
                        self.layers.k_ptrs.data_ptr() + off, self.layers.v_ptrs.data_ptr() + off,
                        err_ptr, stream,
                    ),
                    "mshift_save",
                )
                n += 1
        self.last_launches = n
        return n

    def finish(self, p: Prepared, check: bool) -> None:
        stream = p.stream
        self.staging.finish(p.slot, stream)
        if check:
            _raise_bits(self.staging.read_err(p.slot, stream), f"shift {p.kind}")

    # -- one-call entry points ---------------------------------------------
    def load(self, runs: list[RunSpec], store: StoreView, inv_freq: torch.Tensor, *,
             k_scales: torch.Tensor | None = None, check: bool = True) -> None:
        """Every run x every layer: store rows -> paged cache, K rotated by its delta.

        ``inv_freq`` is the fp32 device tensor of the RoPE inverse frequencies.
        ``k_scales`` (the per-layer K scales of an e4m3 cache) is accepted and
        not needed: the scale cancels.
        """
        if not runs:
            return
        p = self.prepare_load(runs, store, inv_freq, k_scales=k_scales)
        self.launch(p)
        self.finish(p, check)

    def save(self, runs: list[RunSpec], store: StoreView, *, first_layer: int = 0,
             n_layers: int | None = None, check: bool = True, err: int | None = None) -> None:
        """Every run x layers ``[first_layer, +n_layers)``: paged rows -> store rows, bit copy.

        ``store.ptrs`` has one column per layer of that range.  ``err``: see
        :meth:`launch` (only with ``check=False``).
        """
        if not runs:
            return
        p = self.prepare_save(runs, store, first_layer=first_layer, n_layers=n_layers)
        self.launch(p, err=err)
        self.finish(p, check and err is None)
