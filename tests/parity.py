"""Comparison of a cache the kernels wrote with the oracle's (a test helper).

bf16, fp16 and fp32 caches must match the oracle bit for bit.  For e4m3 the
kernels rotate the codes with the layer's scale cancelled (dequantising and
requantising with the same scale) in one fused rounding, where the oracle
follows dequantise -> rotate -> divide step by step; the two agree except next
to an e4m3 rounding boundary, where they are one step apart -- the north
star's FP8 bar.  V rows are copies and must be identical in every dtype.
"""

from __future__ import annotations

import numpy as np

from oracle import shift_oracle as O


def v_mask(paged: O.Paged) -> np.ndarray:
    """True at every element of the flat cache that belongs to a V row."""
    size = paged.flat.size
    n_slots = (size - max(paged.k_base, paged.v_base) + paged.blk - 1) // paged.blk \
        * paged.block_size
    mask = np.zeros(size, dtype=bool)
    mask[paged._index(paged.v_base, np.arange(n_slots))] = True
    return mask


def assert_cache_matches(got_bits: np.ndarray, paged: O.Paged, dtype: str, tag=None) -> None:
    got = np.asarray(got_bits).reshape(-1)
    want = paged.flat
    if dtype != O.E4M3:
        assert np.array_equal(got, want), tag
        return
    vm = v_mask(paged)
    assert np.array_equal(got[vm], want[vm]), ("V", tag)
    steps = O.ulp_distance(got, want, O.E4M3)
    assert steps.max() <= 1, (tag, int(steps.max()))
    assert (steps > 0).mean() < 1e-3, (tag, float((steps > 0).mean()))


def assert_k_codes_match(got_k: np.ndarray, want_k: np.ndarray, dtype: str, tag=None) -> None:
    """K rows alone: exact, or within one e4m3 step."""
    if dtype != O.E4M3:
        assert np.array_equal(got_k, want_k), tag
        return
    steps = O.ulp_distance(got_k, want_k, O.E4M3)
    assert steps.max() <= 1, (tag, int(steps.max()))
    assert (steps > 0).mean() < 1e-3, (tag, float((steps > 0).mean()))


def reference_tables(deltas, inv_freq, device) -> np.ndarray:
    """``[n, 2, half]`` cos/sin tables exactly as the reference's GPU path builds them
    (``src/marathon/shift_kernels.py:73-79``): the fp32 angle ``float(delta) *
    inv_freq`` and torch's fp32 ``cos`` / ``sin`` on the CUDA device.  The oracle
    rotates with these in the GPU tests, so a bit-exact match covers the tables
    and the rotation together."""
    import torch

    inv = torch.as_tensor(np.asarray(inv_freq, dtype=np.float32)).to(device)
    out = []
    for d in deltas:
        ang = float(d) * inv
        out.append(torch.stack((ang.cos(), ang.sin())).cpu().numpy())
    return np.stack(out).astype(np.float32) if out else np.zeros((0, 2, inv.numel()),
                                                                 np.float32)
