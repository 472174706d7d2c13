"""The TMA load kernel's bounded waits: a wait that runs out is reported, not hung.

Every wait in the TMA (``cp.async.bulk``) load kernel is bounded.  When one
runs out the launch sets ``MSHIFT_EBIT_TIMEOUT``, stops writing, waits (with
the normal bound) for the bulk copies it already issued so none is left
writing shared memory, and returns -- the context stays usable.  The
diagnostic hook ``mshift_debug_first_wait(0)`` makes every consumer warp's
first wait give up at once, which exercises exactly that path without any
fault: the copies themselves are ordinary in-bounds copies and complete.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

BS, H, D, L, NBLK = 16, 8, 128, 2, 64


def test_a_timed_out_tma_load_flags_writes_nothing_and_the_next_load_is_exact(cuda):
    from marathon_b200 import _lib
    from marathon_b200.paged import KVLayers
    from marathon_b200.shift_kernels import (Launcher, RunSpec, ShiftError, StoreView, inv_freq,
                                             set_load_kernel)
    from oracle import shift_oracle as O
    from parity import reference_tables

    lib = _lib.load()
    g = torch.Generator().manual_seed(9)
    stores = [torch.randn(400, H, 2 * D, generator=g).to(torch.bfloat16).to(cuda)
              for _ in range(L)]
    kv = [torch.randn(NBLK, BS, H, 2 * D, generator=g).to(torch.bfloat16).to(cuda)
          for _ in range(L)]
    before = [t.clone() for t in kv]
    la = Launcher(KVLayers(kv, BS, "nhd"))
    view = StoreView(np.array([[t.data_ptr() for t in stores]], dtype=np.uint64),
                     np.array([400]), H * 2 * D, 2 * D, stores)
    inv = inv_freq(D, 1e6).to(cuda)
    bt = np.random.default_rng(2).permutation(NBLK).astype(np.int32)
    runs = [RunSpec(0, 10, 300, delta=37, block_table=bt[:24], paged_start=7),
            RunSpec(0, 320, 50, delta=-12, block_table=bt[30:], paged_start=0)]
    prev_kernel = set_load_kernel("bulk")
    try:
        assert lib.mshift_debug_first_wait(0) == -1
        try:
            with pytest.raises(ShiftError, match="did not complete in time"):
                la.load(runs, view, inv, check=True)
        finally:
            assert lib.mshift_debug_first_wait(-1) == 0
        torch.cuda.synchronize()
        for a, b in zip(kv, before, strict=True):  # the aborted launch wrote nothing
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        la.load(runs, view, inv, check=True)  # the same load with normal waits
    finally:
        set_load_kernel(prev_kernel)
    torch.cuda.synchronize()
    for layer in range(L):
        got = kv[layer].cpu().view(torch.int16).numpy().view(np.uint16)
        src = stores[layer].cpu().view(torch.int16).numpy().view(np.uint16)
        for r in runs:
            pos = np.arange(r.paged_start, r.paged_start + r.length)
            at = got[r.block_table[pos // BS], pos % BS]
            rows = src[r.store_start : r.store_start + r.length]
            tab = reference_tables([r.delta], O.inv_freq(D, 1e6), cuda)[0]
            assert np.array_equal(at[..., D:], rows[..., D:])
            assert np.array_equal(at[..., :D], O.shift_k_bits(rows[..., :D], tab, O.BF16))
