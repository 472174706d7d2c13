"""The shift path as PyTorch operators: ``torch.ops.marathon.*``.

Tensor-level entry points over the same native library, for callers that
want PyTorch's operator registry rather than the connector classes (an
operator shows up in profiles and traces under its own name, and
``torch.compile`` treats it as one opaque call that mutates its cache
arguments).  Each operator runs the CUDA kernels and nothing else; CPU tensors
raise.

* ``marathon::scatter_shifted(src, kv!, slots, block_size, hnd, table?)`` --
  the reference's ``scatter_shifted`` (``src/marathon/shift_kernels.py:162-210``)
  with the rotation given as a ``[2, rotary/2]`` cos/sin table (``RopeShift.table``)
  or None for a plain scatter.
* ``marathon::shift_load(stores, kv!, segments, block_tables, inv_freq,
  block_size, layout, k_scales?)`` -- every segment of every session through
  every layer in one launch: the connector's load step
  (``vllm_shift_connector.py:481-534``).
* ``marathon::shift_save(kv, stores!, segments, block_tables, block_size,
  layout)`` -- paged rows back into the store rows at the same positions
  (``vllm_shift_connector.py:539-553``), all layers in one launch.

``stores`` is flat, session-major: session ``s``'s layer ``l`` buffer is
``stores[s * n_layers + l]`` (``[capacity, heads, 2*head_size]``).
``segments`` is an int64 ``[n, 5]`` tensor of ``(session, src_start,
dst_start, length, delta)`` rows on the host; for a save ``src_start`` is
ignored and rows ``[dst_start, +length)`` are written.  ``block_tables[s]`` is
session ``s``'s int32 block table (its logical position ``p`` lives in block
``block_tables[s][p // block_size]``).
"""

from __future__ import annotations

import numpy as np
import torch

from .paged import KVLayers
from .shift_kernels import Launcher, RopeShift, RunSpec, ShiftError, StoreView, scatter_shifted

_launchers: dict = {}


def _launcher(kv: list[torch.Tensor], block_size: int, layout: str) -> Launcher:
    """One launcher per set of cache addresses and shapes (their pointers are staged once).

    The cached launcher keeps only the addresses, not the tensors: a cache the
    caller frees is freed, and a later cache at the same addresses with the
    same shape, strides and dtype is served by the same launcher.
    """
    key = (tuple((t.data_ptr(), tuple(t.shape), t.stride(), t.dtype) for t in kv), block_size,
           layout)
    la = _launchers.get(key)
    if la is None:
        if len(_launchers) > 16:
            for old in _launchers.values():
                old.drain()  # their pinned staging may still feed copies in flight
            _launchers.clear()
        fp8 = kv[0].dtype in (torch.float8_e4m3fn, torch.uint8)
        la = Launcher(KVLayers(list(kv), block_size, layout, fp8=fp8))
        la.layers.tensors = []  # the kernels need the staged addresses only
        _launchers[key] = la
    return la


def _view(stores: list[torch.Tensor], n_layers: int) -> StoreView:
    if not stores or len(stores) % n_layers:
        raise ShiftError(f"{len(stores)} store buffers for {n_layers} layers")
    n_sessions = len(stores) // n_layers
    ptrs = np.array([t.data_ptr() for t in stores], dtype=np.uint64).reshape(n_sessions, n_layers)
    caps = np.array([stores[s * n_layers].shape[0] for s in range(n_sessions)], dtype=np.int64)
    t = stores[0]
    for b in stores:
        if not b.is_cuda or b.stride() != t.stride() or b.dtype != t.dtype:
            raise ShiftError("store buffers must be CUDA tensors of one dtype and row layout")
    return StoreView(ptrs, caps, t.stride(0), t.stride(1), list(stores))


def _runs(segments: torch.Tensor, block_tables: list[torch.Tensor], load: bool) -> list[RunSpec]:
    seg = segments.to("cpu", torch.int64).numpy()
    if seg.ndim != 2 or seg.shape[1] != 5:
        raise ShiftError("segments must be [n, 5]: session, src_start, dst_start, length, delta")
    tables = [bt.to(torch.int32).contiguous() for bt in block_tables]
    runs = []
    for s, src, dst, n, delta in seg.tolist():
        if not 0 <= s < len(tables):
            raise ShiftError(f"segment names session {s} of {len(tables)}")
        bt = tables[s]
        if not bt.is_cuda:
            bt = bt.numpy()  # travels inside the batch's descriptor copy
        runs.append(RunSpec(s, src if load else dst, n, delta if load else 0,
                            block_table=bt, paged_start=dst))
    return runs


@torch.library.custom_op("marathon::scatter_shifted", mutates_args=("kv",))
def _scatter_shifted_op(src: torch.Tensor, kv: torch.Tensor, slots: torch.Tensor,
                        block_size: int, hnd: bool, table: torch.Tensor | None = None) -> None:
    shift = None
    if table is not None:
        tab = table.to(torch.float32).reshape(2, table.shape[-1]).contiguous()
        c, sn = tab[0], tab[1]
        # only `table` (and the rotary width) is read by the kernel path; the
        # delta is any non-zero marker: the table already encodes it
        shift = RopeShift(1, None, None, None, torch.cat((c, c)), torch.cat((sn, sn)), tab)
    scatter_shifted(src, kv, slots, block_size, hnd, shift)


@torch.library.custom_op("marathon::shift_load", mutates_args=("kv",))
def _shift_load_op(stores: list[torch.Tensor], kv: list[torch.Tensor], segments: torch.Tensor,
                   block_tables: list[torch.Tensor], inv_freq: torch.Tensor, block_size: int,
                   layout: str, k_scales: torch.Tensor | None = None) -> None:
    la = _launcher(kv, block_size, layout)
    runs = _runs(segments, block_tables, load=True)
    if runs:
        la.load(runs, _view(stores, len(kv)), inv_freq.to(la.device, torch.float32),
                k_scales=k_scales, check=True)


@torch.library.custom_op("marathon::shift_save", mutates_args=("stores",))
def _shift_save_op(kv: list[torch.Tensor], stores: list[torch.Tensor], segments: torch.Tensor,
                   block_tables: list[torch.Tensor], block_size: int, layout: str) -> None:
    la = _launcher(kv, block_size, layout)
    runs = _runs(segments, block_tables, load=False)
    if runs:
        la.save(runs, _view(stores, len(kv)), check=True)


@_scatter_shifted_op.register_fake
def _(src, kv, slots, block_size, hnd, table=None) -> None:
    return None


@_shift_load_op.register_fake
def _(stores, kv, segments, block_tables, inv_freq, block_size, layout, k_scales=None) -> None:
    return None


@_shift_save_op.register_fake
def _(kv, stores, segments, block_tables, block_size, layout) -> None:
    return None
