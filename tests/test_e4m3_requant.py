"""The e4m3 requantisation shortcut of the load kernel, checked on the CPU.

The kernel forms the code of ``r / s`` (``s`` a per-layer K scale) without
dividing: it converts ``r * idn`` and ``r * iup``, with ``idn`` / ``iup`` the
fp32 roundings of ``fl(1/s) * (1 -+ 2^-21)``, and keeps the code when both
agree, dividing only when they differ.  This restates that arithmetic in
numpy fp32 (every product correctly rounded, as ``__fmul_rn`` /
``__fmul2_rn`` are) and checks that whenever the two ends agree, their code is
the one the oracle defines: ``RNE_e4m3(clamp(fl(r / s), +-448))``.  Quotients
are placed at, and within +-20 ulp of, every rounding boundary of e4m3, plus
random values, for a spread of scales.
"""

from __future__ import annotations

import numpy as np
import torch

DN = np.float32(0.99999952316284180)  # 1 - 2^-21
UP = np.float32(1.00000047683715820)  # 1 + 2^-21


def e4m3_codes(x: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.clip(x, -448, 448).astype(np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def test_interval_ends_agree_only_on_the_exact_code():
    rng = np.random.default_rng(0)
    codes = np.arange(256, dtype=np.uint8)
    vals = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy().astype(np.float64)
    vals = np.unique(vals[np.isfinite(vals)])
    mids = (vals[1:] + vals[:-1]) / 2
    k = np.arange(-20, 21)
    fallback = total = 0
    for s in np.float32(np.concatenate([rng.uniform(0.01, 0.1, 6), [0.01, 0.1, 1.0, 0.3]])):
        inv = np.float32(1) / s
        idn, iup = np.float32(inv * DN), np.float32(inv * UP)
        q = (mids[:, None] * (1 + k[None, :] * 2.0**-24)).reshape(-1)
        r = np.float32(q * np.float64(s))
        r = np.concatenate([r, rng.normal(0, 5, 50_000).astype(np.float32)])
        r = np.concatenate([r, np.nextafter(r, np.float32(np.inf)),
                            np.nextafter(r, np.float32(-np.inf)), -r]).astype(np.float32)
        want = e4m3_codes(r / s)  # numpy's fp32 divide is correctly rounded
        lo, hi = e4m3_codes(r * idn), e4m3_codes(r * iup)
        agree = lo == hi
        assert np.array_equal(lo[agree], want[agree])
        fallback += int((~agree).sum())
        total += r.size
    # the boundary-hugging inputs are built to hit the division path often
    assert 0 < fallback < total // 10
