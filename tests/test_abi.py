"""The C ABI library: it loads, exports every declared symbol, and validates on the host.

Runs without a GPU: only entry points that never reach the CUDA runtime are
called (host helpers, and argument errors that return before any launch).
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from marathon_b200 import _lib
from marathon_b200.build import LIB, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "marathon_shift.h"


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def declared() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"MSHIFT_API\s+[\w\s\*]+?\b(mshift_\w+)\s*\(", text)


def test_header_and_binding_agree():
    assert sorted(declared()) == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(LIB))
    for name in declared():
        assert hasattr(raw, name), name


def test_only_declared_symbols_are_exported(lib):
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True,
                         text=True, check=True).stdout
    mine = sorted(line.split()[-1] for line in out.splitlines() if " mshift_" in line)
    assert mine == sorted(declared())


def test_struct_layouts_match_the_header(lib):
    assert ctypes.sizeof(_lib.Run) == 56
    assert ctypes.sizeof(_lib.Paged) == 48
    assert _lib.Run.tile_begin.offset == 48
    assert _lib.RUN_DTYPE.itemsize == 56


def test_version_and_strerror(lib):
    assert b"sm_100a" in lib.mshift_version()
    assert lib.mshift_strerror(_lib.EINVAL) == b"invalid argument"
    assert lib.mshift_strerror(99) == b"unknown status"


def test_supported_variants(lib):
    assert lib.mshift_supported(_lib.BF16, 128, 128)
    assert lib.mshift_supported(_lib.E4M3, 128, 128)
    assert lib.mshift_supported(_lib.BF16, 256, 64)
    assert not lib.mshift_supported(_lib.BF16, 96, 96)
    assert not lib.mshift_supported(7, 128, 128)


def test_default_tile_tokens(lib):
    assert lib.mshift_default_tile_tokens(8) == 32
    assert lib.mshift_default_tile_tokens(1) == 256
    assert lib.mshift_default_tile_tokens(64) == 16


def test_plan_tiles_prefix(lib):
    runs = (_lib.Run * 3)()
    for r, n in zip(runs, (100, 32, 1), strict=True):
        r.len = n
    total = lib.mshift_plan_tiles(ctypes.cast(runs, ctypes.c_void_p), 3, 32)
    assert total == 4 + 1 + 1
    assert [r.tile_begin for r in runs] == [0, 4, 5]
    runs[1].len = 0
    assert lib.mshift_plan_tiles(ctypes.cast(runs, ctypes.c_void_p), 3, 32) == -1


def test_argument_errors_return_before_any_launch(lib):
    p = _lib.Paged(4096, 2048, 256, 10, 16, 8, 128, _lib.BF16)
    # null runs / zero layers / bad tile size
    assert lib.mshift_load(p, 128, None, 1, 32, 1, 1, 8, 8, 1, 2048, 256, 8, 8, None, 0, None,
                           8, None) == _lib.EINVAL
    assert lib.mshift_load(p, 128, 16, 1, 0, 1, 1, 8, 8, 1, 2048, 256, 8, 8, None, 0, None,
                           8, None) == _lib.EINVAL
    assert lib.mshift_save(p, 16, 1, 32, 1, 0, 8, 8, 1, 2048, 256, 8, 8, 8, None) == _lib.EINVAL
    # tiles of more than 512 tokens
    assert lib.mshift_load(p, 128, 16, 1, 513, 1, 1, 8, 8, 1, 2048, 256, 8, 8, None, 0, None,
                           8, None) == _lib.EINVAL
    assert lib.mshift_save(p, 16, 1, 513, 1, 1, 8, 8, 1, 2048, 256, 8, 8, 8, None) == _lib.EINVAL
    # strides that are not whole 16-byte vectors
    bad = _lib.Paged(4096, 2048, 255, 10, 16, 8, 128, _lib.BF16)
    assert lib.mshift_save(bad, 16, 1, 32, 1, 1, 8, 8, 1, 2048, 256, 8, 8, 8, None) == _lib.EINVAL
    # an uncompiled head geometry
    odd = _lib.Paged(4096, 2048, 256, 10, 16, 8, 96, _lib.BF16)
    assert lib.mshift_load(odd, 96, 16, 1, 32, 1, 1, 8, 8, 1, 2048, 256, 8, 8, None, 0, None,
                           8, None) == _lib.EUNSUPPORTED
    # rotation tables announced (n_tables = 1) but not passed
    f8 = _lib.Paged(4096, 2048, 256, 10, 16, 8, 128, _lib.E4M3)
    assert lib.mshift_load(f8, 128, 16, 1, 32, 1, 1, 8, 8, 1, 2048, 256, 8, 8, None, 1, None,
                           8, None) == _lib.EINVAL
    # zero-length single scatter is a successful no-op
    assert lib.mshift_scatter_shifted(None, 0, 0, 0, None, None, p, None, None, 128, None, None,
                                      None) == _lib.OK
    # negative sizes
    assert lib.mshift_rope_tables(None, -1, None, 64, None, None) == _lib.EINVAL


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(_lib.ShiftError, match="not built"):
        _lib.load()


def test_stage_validates_before_touching_cuda(lib):
    """``mshift_stage`` rejects malformed copy lists on the host (no CUDA call is
    made for them, nor for empty or zero-byte lists)."""
    import numpy as np

    assert _lib.COPY_DTYPE.itemsize == 24  # mshift_copy: dst, src, bytes
    assert lib.mshift_stage(None, 0, None) == _lib.OK
    assert lib.mshift_stage(None, 1, None) == _lib.EINVAL
    assert lib.mshift_stage(None, -1, None) == _lib.EINVAL
    rec = np.zeros(2, dtype=_lib.COPY_DTYPE)
    assert lib.mshift_stage(rec.ctypes.data, 2, None) == _lib.OK  # zero-byte ranges skipped
    rec[1]["bytes"] = -16
    assert lib.mshift_stage(rec.ctypes.data, 2, None) == _lib.EINVAL
    rec[1] = (0, 4096, 16)  # bytes with a null destination
    assert lib.mshift_stage(rec.ctypes.data, 2, None) == _lib.EINVAL


def test_status_flags_match_the_header():
    """Every MSHIFT_EBIT_* flag of the header has the same value in the binding."""
    text = (Path(__file__).resolve().parents[1] / "include" / "marathon_shift.h").read_text()
    flags = {m[1]: int(m[2]) for m in re.finditer(r"#define MSHIFT_EBIT_(\w+) (\d+)u", text)}
    assert flags == {"SLOT": 1, "STORE": 2, "SESSION": 4, "TABLE": 8, "TIMEOUT": 16, "CLAIM": 32}
    for name, value in flags.items():
        assert getattr(_lib, f"EBIT_{name}") == value
        assert _lib.describe_bits(value) != "none"
    assert max(flags.values()) < 256  # the low 8 bits; bits 8..31 carry the claim count
