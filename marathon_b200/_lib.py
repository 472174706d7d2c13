"""ctypes binding of ``libmarathon_shift.so`` (the C ABI in ``include/marathon_shift.h``).

This module is the only place Python touches the native library.  It never
falls back to anything: if the library is missing or a call returns an error,
it raises.  The structures below mirror the header byte for byte, and
:data:`RUN_DTYPE` is the same ``mshift_run`` layout as a numpy structured dtype
so that a batch of run descriptors can be packed without a Python loop.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libmarathon_shift.so"

OK, EINVAL, EUNSUPPORTED, ECUDA, ETOOBIG = 0, 1, 2, 3, 4
EBIT_SLOT, EBIT_STORE, EBIT_SESSION, EBIT_TABLE, EBIT_TIMEOUT, EBIT_CLAIM = 1, 2, 4, 8, 16, 32
BF16, F16, F32, E4M3 = 0, 1, 2, 3
KERNEL_LSU, KERNEL_BULK, KERNEL_AUTO = 0, 1, 2

#: every symbol the header declares; tests check the library exports them all
EXPORTS = (
    "mshift_rope_tables",
    "mshift_scatter_shifted",
    "mshift_load",
    "mshift_save",
    "mshift_plan_tiles",
    "mshift_default_tile_tokens",
    "mshift_supported",
    "mshift_version",
    "mshift_strerror",
    "mshift_last_cuda_error",
    "mshift_load_noalloc",
    "mshift_noalloc_max_deltas",
    "mshift_set_load_kernel",
    "mshift_debug_first_wait",
    "mshift_stage",
    "mshift_enable_peer",
)


class Paged(ctypes.Structure):
    """``mshift_paged``: geometry of one layer of the paged KV cache."""

    _fields_ = [
        ("blk_stride", ctypes.c_int64),
        ("off_stride", ctypes.c_int64),
        ("head_stride", ctypes.c_int64),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class Run(ctypes.Structure):
    """``mshift_run``: one run of tokens between a store and the paged cache."""

    _fields_ = [
        ("store_start", ctypes.c_int64),
        ("paged_start", ctypes.c_int64),
        ("slots", ctypes.c_uint64),
        ("block_table", ctypes.c_uint64),
        ("block_table_len", ctypes.c_int32),
        ("len", ctypes.c_int32),
        ("session", ctypes.c_int32),
        ("table", ctypes.c_int32),
        ("tile_begin", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


RUN_DTYPE = np.dtype(
    [
        ("store_start", "<i8"),
        ("paged_start", "<i8"),
        ("slots", "<u8"),
        ("block_table", "<u8"),
        ("block_table_len", "<i4"),
        ("len", "<i4"),
        ("session", "<i4"),
        ("table", "<i4"),
        ("tile_begin", "<i4"),
        ("reserved", "<i4"),
    ]
)
assert RUN_DTYPE.itemsize == ctypes.sizeof(Run) == 56

#: ``mshift_copy``: one staged range (dst, src, bytes)
COPY_DTYPE = np.dtype([("dst", "<u8"), ("src", "<u8"), ("bytes", "<i8")])

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64

_SIGNATURES = {
    "mshift_rope_tables": (ctypes.c_int, [_P, _I32, _P, _I32, _P, _P]),
    "mshift_scatter_shifted": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _P, _P, ctypes.POINTER(Paged), _P, _P, _I32, _P, _P, _P],
    ),
    "mshift_load": (
        ctypes.c_int,
        [ctypes.POINTER(Paged), _I32, _P, _I32, _I32, _I32, _I32, _P, _P, _I32, _I64, _I64,
         _P, _P, _P, _I32, _P, _P, _P],
    ),
    "mshift_save": (
        ctypes.c_int,
        [ctypes.POINTER(Paged), _P, _I32, _I32, _I32, _I32, _P, _P, _I32, _I64, _I64, _P, _P,
         _P, _P],
    ),
    "mshift_plan_tiles": (_I32, [_P, _I32, _I32]),
    "mshift_default_tile_tokens": (_I32, [_I32]),
    "mshift_supported": (ctypes.c_int, [_I32, _I32, _I32]),
    "mshift_version": (ctypes.c_char_p, []),
    "mshift_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "mshift_last_cuda_error": (ctypes.c_char_p, []),
    "mshift_load_noalloc": (
        ctypes.c_int,
        [ctypes.POINTER(Paged), _I32, _P, _I32, _I32, _I32, _I32, _P, _P, _I32, _I64, _I64,
         _P, _P, _P, _I32, _P, _P, _P, _P],
    ),
    "mshift_noalloc_max_deltas": (_I32, []),
    "mshift_set_load_kernel": (ctypes.c_int, [ctypes.c_int]),
    "mshift_debug_first_wait": (_I32, [_I32]),
    "mshift_stage": (ctypes.c_int, [_P, _I32, _P]),
    "mshift_enable_peer": (ctypes.c_int, [_I32]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class ShiftError(RuntimeError):
    """A native entry point returned a non-zero status, or a kernel flagged bad input."""


def load() -> ctypes.CDLL:
    """The loaded library with typed entry points. Raises if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ShiftError(
                    f"{LIB_PATH.name} is not built; run `python -m marathon_b200.build` "
                    "(there is no non-CUDA implementation of the shift path)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    """Raise :class:`ShiftError` for a non-zero status from ``what``."""
    if status == OK:
        return
    lib = load()
    msg = lib.mshift_strerror(status).decode()
    if status == ECUDA:
        msg += f" ({lib.mshift_last_cuda_error().decode()})"
    raise ShiftError(f"{what}: {msg}")


def describe_bits(bits: int) -> str:
    """Names of the ``MSHIFT_EBIT_*`` flags in a status word (its low 8 bits;
    bits 8..31 are the tile-claim count a batched launch uses while it runs)."""
    bits &= 0xFF
    names = []
    for bit, name in (
        (EBIT_SLOT, "slot outside the paged cache"),
        (EBIT_STORE, "store position outside the session buffer"),
        (EBIT_SESSION, "bad session index or missing store buffer"),
        (EBIT_TABLE, "bad rotation-table index"),
        (EBIT_TIMEOUT, "a bulk copy did not complete in time; the launch stopped early"),
        (EBIT_CLAIM, "the tile-claim counter went backwards (status word shared with a "
                     "launch in flight); the launch stopped early"),
    ):
        if bits & bit:
            names.append(name)
    return ", ".join(names) or "none"
