"""Descriptor staging ring: batches prepared while earlier ones are still queued.

A launcher packs each batch's descriptors into one of its pinned staging slots
and copies them to the device, by default on its own copy stream ahead of the
launch stream (``Launcher.EARLY_UPLOAD``).  A slot may be refilled only once
the batch that last used it -- its descriptor copy and its kernels -- has
finished.  Here the launch stream is held by a long queued kernel while more
batches than slots are prepared, so every reuse of a slot happens while its
previous batch is still waiting; each batch writes its own blocks with its own
delta and block table (which rides in the descriptor copy), so a descriptor
overwritten too early would land rows in the wrong place.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

BS, H, D, L, NBLK, BATCHES = 16, 8, 128, 3, 200, 5


def _run_batches(cuda, early: bool, monkeypatch):
    from marathon_b200.paged import KVLayers
    from marathon_b200.shift_kernels import Launcher, RunSpec, StoreView, inv_freq

    monkeypatch.setattr(Launcher, "EARLY_UPLOAD", early)
    g = torch.Generator().manual_seed(3)
    stores = [torch.randn(512, H, 2 * D, generator=g).to(torch.bfloat16).to(cuda)
              for _ in range(L)]
    kv = [torch.zeros(NBLK, BS, H, 2 * D, dtype=torch.bfloat16, device=cuda) for _ in range(L)]
    la = Launcher(KVLayers(kv, BS, "nhd"), staging_slots=2)
    view = StoreView(np.array([[t.data_ptr() for t in stores]], dtype=np.uint64),
                     np.array([512]), H * 2 * D, 2 * D, stores)
    inv = inv_freq(D, 1e6).to(cuda)
    bt = np.random.default_rng(0).permutation(NBLK).astype(np.int32)
    torch.cuda._sleep(100_000_000)  # a bounded spin of ~50 ms ahead of every batch
    for b in range(BATCHES):
        run = RunSpec(0, 64 * b, 64, delta=17 * (b + 1) - 40,
                      block_table=bt[40 * b : 40 * b + 40].copy(), paged_start=0)
        la.load([run], view, inv, check=False)
    torch.cuda.synchronize()
    la.drain()
    return ([t.cpu().view(torch.int16).numpy().view(np.uint16) for t in kv],
            [t.cpu().view(torch.int16).numpy().view(np.uint16) for t in stores], bt)


@pytest.mark.gpu
def test_early_upload_with_more_batches_than_slots_behind_a_busy_stream(cuda, monkeypatch):
    from oracle import shift_oracle as O
    from parity import reference_tables

    early, stores, bt = _run_batches(cuda, True, monkeypatch)
    late, _, _ = _run_batches(cuda, False, monkeypatch)
    for a, b in zip(early, late, strict=True):
        assert np.array_equal(a, b)
    inv = O.inv_freq(D, 1e6)
    for b in range(BATCHES):
        tab = reference_tables([17 * (b + 1) - 40], inv, cuda)[0]
        pos = np.arange(64)
        blk = bt[40 * b : 40 * b + 40][pos // BS]
        for layer in range(L):
            src = stores[layer][64 * b : 64 * b + 64]
            got = early[layer][blk, pos % BS]
            assert np.array_equal(got[..., D:], src[..., D:])
            assert np.array_equal(got[..., :D], O.shift_k_bits(src[..., :D], tab, O.BF16))
