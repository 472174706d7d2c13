"""The e4m3 load arithmetic, checked on the CPU against the oracle's definition.

The oracle defines an e4m3 re-rotation as dequantise -> rotate -> requantise:
``x = code * s`` (fp32), the fp32 rotation of ``x``, ``/ s``, saturate to
+-448, round to the nearest e4m3 code (ties to even).  With one scale ``s``
per layer for both directions the scale cancels, and the load kernels compute
``RNE(sat(fma(x, c, -fl(y * sn))))`` (``rb = fma(y, c, fl(x * sn))``) directly
on the codes' values.  Both fp32 results lie within a few fp32 ulps of the
terms (``|code| <= 448``) of the exact rotation, far closer together than the
smallest e4m3 step (2^-9), so their codes can differ by at most one step,
and only next to a rounding boundary.

This restates the kernel's arithmetic in numpy (products of two fp32 values
are exact in float64; the fused add is rounded once to fp32 from float64 --
a double rounding that can only move a result that sits exactly on an fp32
tie, far below the e4m3 resolution) and checks the one-step bound on every
code pair against tables of several deltas, plus the share of codes that
differ at all.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import shift_oracle as O


def _kernel_model(x_codes: np.ndarray, y_codes: np.ndarray, c: np.ndarray, s: np.ndarray):
    x = O.e4m3_to_f32(x_codes).astype(np.float64)
    y = O.e4m3_to_f32(y_codes).astype(np.float64)
    c, s = c.astype(np.float64), s.astype(np.float64)
    ys = (y * s).astype(np.float32).astype(np.float64)
    xs = (x * s).astype(np.float32).astype(np.float64)
    ra = (x * c - ys).astype(np.float32)
    rb = (y * c + xs).astype(np.float32)
    return O.f32_to_e4m3(ra), O.f32_to_e4m3(rb)


def test_scale_cancelled_rotation_is_within_one_step_of_the_oracle():
    codes = np.arange(256, dtype=np.uint8)
    codes = codes[(codes & 0x7F) != 0x7F]  # no NaN codes
    xa, ya = np.meshgrid(codes, codes, indexing="ij")
    xa, ya = xa.reshape(-1), ya.reshape(-1)  # every (code, partner code) pair
    inv = O.inv_freq(128, 1e6)
    rng = np.random.default_rng(3)
    differ = total = 0
    for delta in (180, -566, 37, 6759):
        table = O.rope_tables([delta], inv)[0]
        for i in rng.choice(64, 6, replace=False):
            c = np.full(xa.shape, table[0, i], np.float32)
            s = np.full(xa.shape, table[1, i], np.float32)
            ka, kb = _kernel_model(xa, ya, c, s)
            for scale in (0.01, 0.0371, 0.1):
                # the oracle on the partner pair: K row [x | y] with a 1-entry table
                rows = np.stack((xa, ya), axis=-1)
                tab = np.stack((table[0, i : i + 1], table[1, i : i + 1]))
                want = O.shift_k_bits(rows, tab, O.E4M3, scale)
                for got, w in ((ka, want[:, 0]), (kb, want[:, 1])):
                    steps = O.ulp_distance(got, w, O.E4M3)
                    assert steps.max() <= 1, (delta, i, scale)
                    differ += int((steps > 0).sum())
                    total += steps.size
    assert differ < total * 1e-3


def test_saturation_matches_torch_clamped_conversion():
    r = np.array([447.9, 448.0, 460.0, 10_000.0, -10_000.0, -449.0], dtype=np.float32)
    want = torch.from_numpy(np.clip(r, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8)
    assert np.array_equal(O.f32_to_e4m3(r), want.numpy())
