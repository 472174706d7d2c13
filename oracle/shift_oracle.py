"""CPU oracle of the position-shifted KV reuse path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference leg
import it.  The package ``marathon_b200`` never does, and has no CPU path.

It restates, in numpy, the reference's algorithm for the path
(acrosley/marathon, paths relative to that project):

* ``inv_freq``        src/marathon/vllm_shift_connector.py:196-198
* ``rope_tables``     src/marathon/shift_kernels.py:68-84 (angle ``float(delta) *
                      inv_freq`` in fp32, then cos / sin)
* ``rotate_keys``     src/marathon/shift_kernels.py:150-156 (torch path: fp32
                      ``k*cos + rotate_half(k)*sin``, each product rounded, then
                      the sum), partial rotary as src/marathon/kvshift_hybrid.py:72-84
* ``slots``           src/marathon/shift_store.py:56-60
* ``scatter_shifted`` src/marathon/shift_kernels.py:141-159 and the Triton kernel
                      :89-132 (K rotated, V copied, paged via strides)
* ``load``            the per-load, per-layer loop of
                      src/marathon/vllm_shift_connector.py:495-518
* ``save``            src/marathon/vllm_shift_connector.py:418-442 + :546-553 and
                      src/marathon/shift_store.py:225-236

Numbers are carried as raw bits (uint16 for bf16/f16, uint8 for e4m3, float32
for fp32) so comparisons against the CUDA path are bit comparisons.

Parity pin: ``tests/test_oracle_golden.py`` checks every function here against
vectors produced by the reference itself (``tests/golden/make_golden.py``
imports the reference's ``marathon`` package and records its outputs) and
against the reference's own known-answer tests.

Two places where this restatement fixes what the reference leaves to its
runtime, both checked against the reference's outputs:

* cos / sin are the correctly rounded fp32 values of the fp32 angle (computed
  in float64, rounded once).  torch's fp32 ``cos`` is within 1 ulp of that;
  the golden test records how many table entries differ.
* e4m3 requantisation (the reference has no scale handling; it casts the fp32
  result straight to the cache dtype, shift_kernels.py:128,156): ``code *
  scale`` -> rotate -> ``/ scale`` -> clamp to +-448 -> round to nearest even.
"""

from __future__ import annotations

import numpy as np

BF16, F16, F32, E4M3 = "bf16", "f16", "f32", "e4m3"
E4M3_MAX = 448.0


# --------------------------------------------------------------- conversions
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 bits, nearest-even; NaN -> 0x7FC0 (torch's c10 rule)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r)


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def _e4m3_magnitudes() -> np.ndarray:
    """Values of codes 0..126 (0x7F is NaN in float8_e4m3fn), increasing."""
    c = np.arange(127, dtype=np.int64)
    e = c >> 3
    m = c & 7
    return np.where(e == 0, m * 2.0**-9, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))


_E4M3 = _e4m3_magnitudes()


def _e4m3_values() -> np.ndarray:
    """fp32 value of every code 0..255 (0x7F, 0xFF: NaN)."""
    mag = np.append(_E4M3, np.nan).astype(np.float32)
    return np.concatenate((mag, -mag)).astype(np.float32)


_E4M3_F32 = _e4m3_values()


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    return _E4M3_F32[np.asarray(codes, dtype=np.uint8)]


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """Saturate to +-448 then round to the nearest e4m3fn code, ties to even.

    Integer arithmetic on the fp32 bit pattern: at or above 2**-6 (e4m3's
    smallest normal) the 24-bit significand is rounded to 4 bits (hidden bit
    plus 3), carrying into the exponent on overflow; below it the value is a
    multiple of 2**-9 and ``rint(|x| * 2**9)`` (exact scaling, ties to even) is
    the code.  Pinned against torch's own conversion by the golden vectors.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x), np.float32(E4M3_MAX))
    u = a.view(np.int32)
    e = (u >> 23) - 127  # unbiased exponent of a normal fp32
    sig = (u & 0x7FFFFF) | 0x800000
    q = sig >> 20
    rem = sig & 0xFFFFF
    q += (rem > 0x80000) | ((rem == 0x80000) & ((q & 1) == 1))
    carry = q >> 4  # 1.111 rounded up to 10.000
    normal = ((e + carry + 7) << 3) | ((q >> carry) & 7)
    sub = np.rint(a * np.float32(2.0**9)).astype(np.int32)  # exact scaling below 2**-6
    code = np.where(a >= np.float32(2.0**-6), normal, sub).astype(np.uint8)
    code = np.where(np.signbit(x), code | np.uint8(0x80), code).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x7F), code)


def _f32_to_e4m3_by_search(x: np.ndarray) -> np.ndarray:
    """Nearest code by search over the 127 magnitudes (the definition; slow)."""
    x = np.asarray(x, dtype=np.float32)
    neg = np.signbit(x)
    a = np.minimum(np.abs(x).astype(np.float64), E4M3_MAX)
    hi = np.clip(np.searchsorted(_E4M3, a, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    d_hi = _E4M3[hi] - a
    d_lo = a - _E4M3[lo]
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(neg, code | 0x80, code).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x7F), code)


def to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == BF16:
        return bf16_to_f32(bits)
    if dtype == F16:
        return f16_to_f32(bits)
    if dtype == F32:
        return np.asarray(bits, dtype=np.float32)
    if dtype == E4M3:
        return e4m3_to_f32(bits)
    raise ValueError(dtype)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == BF16:
        return f32_to_bf16(x)
    if dtype == F16:
        return f32_to_f16(x)
    if dtype == F32:
        return np.asarray(x, dtype=np.float32)
    if dtype == E4M3:
        return f32_to_e4m3(x)
    raise ValueError(dtype)


# -------------------------------------------------------------------- RoPE
def inv_freq(rotary: int, theta: float) -> np.ndarray:
    """``1 / theta ** (arange(0, rotary, 2) / rotary)`` in fp32 (connector :196-198).

    The exponent is formed in fp32 as torch forms it; the power is rounded
    once from float64.
    """
    e = np.arange(0, rotary, 2, dtype=np.float32) / np.float32(rotary)
    p = np.power(np.float64(theta), e.astype(np.float64)).astype(np.float32)
    return (np.float32(1.0) / p).astype(np.float32)


def rope_angles(delta: int, inv: np.ndarray) -> np.ndarray:
    """``float(delta) * inv_freq`` in fp32 (shift_kernels.py:73)."""
    return (np.float32(delta) * np.asarray(inv, dtype=np.float32)).astype(np.float32)


def rope_tables(deltas, inv: np.ndarray) -> np.ndarray:
    """``[n, 2, half]``: cos then sin of each delta's fp32 angles, correctly rounded."""
    deltas = np.atleast_1d(np.asarray(deltas, dtype=np.int64))
    out = np.empty((deltas.size, 2, np.asarray(inv).size), dtype=np.float32)
    for i, d in enumerate(deltas):
        ang = rope_angles(int(d), inv).astype(np.float64)
        out[i, 0] = np.cos(ang).astype(np.float32)
        out[i, 1] = np.sin(ang).astype(np.float32)
    return out


def branchless_tables(table: np.ndarray, head_size: int):
    """The reference's ``cos``/``sgn``/``partner`` form of a ``[2, half]`` table (:74-82)."""
    half = table.shape[1]
    rotary = 2 * half
    cos = np.ones(head_size, dtype=np.float32)
    sgn = np.zeros(head_size, dtype=np.float32)
    cos[:rotary] = np.concatenate([table[0], table[0]])
    sgn[:half] = -table[1]
    sgn[half:rotary] = table[1]
    partner = np.arange(head_size, dtype=np.int32)
    partner[:half] += half
    partner[half:rotary] -= half
    return cos, sgn, partner


def rotate_keys(k: np.ndarray, table: np.ndarray) -> np.ndarray:
    """fp32 re-rotation of ``k[..., D]`` by a ``[2, half]`` table.

    ``out[i] = k[i]*c[i] - k[i+h]*s[i]``, ``out[i+h] = k[i+h]*c[i] + k[i]*s[i]``
    for ``i < h``: each product rounded to fp32, then the sum — the torch
    path's ``kf*emb_cos + cat(-kf[h:], kf[:h])*emb_sin`` term for term.
    Dimensions ``>= 2h`` pass through untouched.
    """
    k = np.asarray(k, dtype=np.float32)
    h = table.shape[1]
    c, s = table[0].astype(np.float32), table[1].astype(np.float32)
    x, y = k[..., :h], k[..., h : 2 * h]
    out = k.copy()
    out[..., :h] = (x * c).astype(np.float32) - (y * s).astype(np.float32)
    out[..., h : 2 * h] = (y * c).astype(np.float32) + (x * s).astype(np.float32)
    return out


def shift_k_bits(k_bits: np.ndarray, table: np.ndarray | None, dtype: str, k_scale: float = 1.0):
    """Rotate K rows given as bits; returns bits of the cache dtype.

    ``table=None`` (delta 0 / no shift) is a bit copy.  E4M3: dequantise with
    ``k_scale``, rotate, divide by ``k_scale``, saturate, round.
    """
    if table is None:
        return np.array(k_bits, copy=True)
    x = to_f32(k_bits, dtype)
    if dtype == E4M3:
        s = np.float32(k_scale)
        x = (x * s).astype(np.float32)
        r = rotate_keys(x, table)
        return f32_to_e4m3((r / s).astype(np.float32))
    return from_f32(rotate_keys(x, table), dtype)


# -------------------------------------------------------------- paged index
def slots(block_ids, lo: int, hi: int, block_size: int) -> np.ndarray:
    """``table[p // bs] * bs + p % bs`` for ``p`` in ``[lo, hi)`` (shift_store.py:56-60)."""
    pos = np.arange(lo, hi, dtype=np.int64)
    table = np.asarray(block_ids, dtype=np.int64)
    return table[pos // block_size] * block_size + pos % block_size


class Paged:
    """A paged cache as one flat bit array plus (K base, V base, strides) in elements."""

    def __init__(self, flat, k_base, v_base, blk, off, head, block_size, heads, head_size):
        self.flat = flat
        self.k_base, self.v_base = int(k_base), int(v_base)
        self.blk, self.off, self.head = int(blk), int(off), int(head)
        self.block_size, self.heads, self.head_size = int(block_size), int(heads), int(head_size)

    @property
    def num_slots(self) -> int:
        return (self.flat.size - max(self.k_base, self.v_base)) // self.blk * self.block_size

    def _index(self, base: int, slot: np.ndarray) -> np.ndarray:
        slot = np.asarray(slot, dtype=np.int64)
        row = (slot // self.block_size) * self.blk + (slot % self.block_size) * self.off
        h = np.arange(self.heads, dtype=np.int64) * self.head
        e = np.arange(self.head_size, dtype=np.int64)
        return base + row[:, None, None] + h[None, :, None] + e[None, None, :]

    def read(self, slot: np.ndarray):
        """(K, V) rows ``[n, heads, head_size]`` at ``slot``."""
        return self.flat[self._index(self.k_base, slot)], self.flat[self._index(self.v_base, slot)]

    def write(self, slot: np.ndarray, k: np.ndarray, v: np.ndarray) -> None:
        self.flat[self._index(self.k_base, slot)] = k
        self.flat[self._index(self.v_base, slot)] = v


def scatter_shifted(src: np.ndarray, paged: Paged, slot: np.ndarray, table, dtype: str,
                    k_scale: float = 1.0) -> None:
    """Write ``src`` (``[n, heads, 2*D]`` bits) to ``slot`` with K rotated (a3/a5)."""
    d = paged.head_size
    paged.write(slot, shift_k_bits(src[..., :d], table, dtype, k_scale), src[..., d:])


def block_table_slots(block_table, paged_start: int, n: int, block_size: int) -> np.ndarray:
    return slots(block_table, paged_start, paged_start + n, block_size)


def load(store, runs, paged_layers, tables, dtype: str, k_scales=None) -> None:
    """Every run, every layer: store rows -> paged, K rotated by its run's table.

    ``store[session][layer]`` is a ``[cap, heads, 2*D]`` bit array;
    ``runs`` are dicts with ``session, store_start, len, table`` and either
    ``slots`` or ``block_table`` + ``paged_start``; ``tables[r["table"]]`` is a
    ``[2, half]`` table or ``table == -1`` for no rotation.  Runs are applied in
    order, layer by layer — the reference's load loop.
    """
    for li, paged in enumerate(paged_layers):
        for r in runs:
            n = int(r["len"])
            sl = run_slots(r, n, paged.block_size)
            rows = store[r["session"]][li][r["store_start"] : r["store_start"] + n]
            tab = tables[r["table"]] if r.get("table", -1) >= 0 else None
            ks = 1.0 if k_scales is None else float(k_scales[li])
            scatter_shifted(rows, paged, sl, tab, dtype, ks)


def save(store, runs, paged_layers) -> None:
    """Every run, every layer: paged rows -> store rows, bit copy."""
    for li, paged in enumerate(paged_layers):
        for r in runs:
            n = int(r["len"])
            sl = run_slots(r, n, paged.block_size)
            k, v = paged.read(sl)
            a = int(r["store_start"])
            d = paged.head_size
            store[r["session"]][li][a : a + n, :, :d] = k
            store[r["session"]][li][a : a + n, :, d:] = v


def run_slots(r: dict, n: int, block_size: int) -> np.ndarray:
    if r.get("slots") is not None:
        return np.asarray(r["slots"], dtype=np.int64)[:n]
    return block_table_slots(r["block_table"], int(r["paged_start"]), n, block_size)


def ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray, dtype: str) -> np.ndarray:
    """Distance in units of the format's spacing, via monotone integer codes."""

    def ordered(bits):
        if dtype in (BF16, F16):
            u = np.asarray(bits, dtype=np.uint16).astype(np.int64)
            return np.where(u & 0x8000, 0x8000 - u, u)
        if dtype == E4M3:
            u = np.asarray(bits, dtype=np.uint8).astype(np.int64)
            return np.where(u & 0x80, 0x80 - u, u)
        u = np.asarray(bits, dtype=np.float32).view(np.uint32).astype(np.int64)
        return np.where(u & 0x80000000, 0x80000000 - u, u)

    return np.abs(ordered(a_bits) - ordered(b_bits))


# ------------------------------------------------------------ tolerance bar
#: stored mantissa bits and smallest normal exponent of each cache format
_FORMAT = {BF16: (7, -126), F16: (10, -14), F32: (23, -126), E4M3: (3, -6)}


def ulp_of(r: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of ``dtype`` at each real value ``r``: ``2**(e - m)`` for ``|r|`` in
    ``[2**e, 2**(e+1))`` with ``m`` stored mantissa bits, the subnormal spacing
    below the smallest normal binade.  E4M3 values are taken after saturation."""
    m, emin = _FORMAT[dtype]
    a = np.abs(np.asarray(r, dtype=np.float64))
    if dtype == E4M3:
        a = np.minimum(a, E4M3_MAX)
    _, e = np.frexp(a)  # a = f * 2**e, 0.5 <= f < 1 (e = 0 at a = 0)
    e = np.where(a > 0, e - 1, emin)
    return np.ldexp(1.0, np.maximum(e, emin) - m)


def within_one_step(got_bits: np.ndarray, r: np.ndarray, dtype: str) -> np.ndarray:
    """True where the stored value is within one unit in the last place of the
    cache format (one e4m3 step for E4M3) of the fp32 result ``r`` -- the bar
    the north star sets: 1 bf16 ulp, or 1 e4m3 step, of the fp32 rotation."""
    r = np.asarray(r, dtype=np.float64)
    if dtype == E4M3:
        r = np.clip(r, -E4M3_MAX, E4M3_MAX)
    got = to_f32(got_bits, dtype).astype(np.float64)
    return np.abs(got - r) <= ulp_of(r, dtype)
