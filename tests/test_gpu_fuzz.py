"""Randomised batches through the C ABI against the oracle.

Each seed draws a geometry (layout, dtype, heads, head size), a handful of
sessions with their own block tables and store capacities, and runs of random
length, offset and delta (some as flat slot lists, some on block tables, some
delta 0), so tile edges, block boundaries, partial last tiles and many-run
batches all occur; both load kernels must land the oracle's bits, and the save
must gather them back.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from marathon_b200 import shift_kernels as sk
from marathon_b200.paged import KVLayers, describe
from marathon_b200.shift_kernels import Launcher, RunSpec, StoreView
from oracle import shift_oracle as O
from parity import assert_cache_matches, reference_tables

pytestmark = pytest.mark.gpu

TORCH_OF = {O.BF16: torch.bfloat16, O.F16: torch.float16, O.F32: torch.float32,
            O.E4M3: torch.float8_e4m3fn}
SHAPES = {"nhd": lambda nb, bs, h, d: (nb, bs, h, 2 * d),
          "hnd": lambda nb, bs, h, d: (nb, h, bs, 2 * d),
          "split": lambda nb, bs, h, d: (2, nb, bs, h, d),
          "split_blocks": lambda nb, bs, h, d: (nb, 2, bs, h, d)}
GEOMETRIES = [(O.BF16, 128, 128), (O.BF16, 64, 64), (O.BF16, 256, 64), (O.F16, 128, 128),
              (O.F32, 128, 128), (O.E4M3, 128, 128), (O.BF16, 128, 64)]


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    if t.dtype == torch.float32:
        return t.numpy()  # the oracle takes fp32 values; comparisons use the bytes
    return t.view(torch.int16).numpy().view(np.uint16)


def _rand(shape, dtype, g):
    x = torch.randn(shape, generator=g)
    if dtype == O.E4M3:
        return (x * 20).clamp(-448, 448).to(torch.float8_e4m3fn)
    return x.to(TORCH_OF[dtype])


@pytest.mark.parametrize("kernel", ["lsu", "bulk"])
@pytest.mark.parametrize("seed", range(8))
def test_random_batches_match_the_oracle(cuda, seed, kernel):
    rng = np.random.default_rng(seed)
    g = torch.Generator().manual_seed(seed)
    dtype, d, rot = GEOMETRIES[seed % len(GEOMETRIES)]
    layout = ["nhd", "hnd", "split", "split_blocks"][seed % 4]
    heads = int(rng.choice([1, 2, 4, 8]))
    bs = int(rng.choice([16, 32]))
    layers = int(rng.integers(1, 4))
    n_sessions = int(rng.integers(1, 5))

    # disjoint destination blocks per session; runs of a session never overlap
    blocks_per = 24
    nblk = n_sessions * blocks_per + 3
    perm = rng.permutation(nblk).astype(np.int32)
    runs_o, runs, caps = [], [], []
    for s in range(n_sessions):
        table = perm[s * blocks_per : (s + 1) * blocks_per]
        cap = int(rng.integers(300, 900))
        caps.append(cap)
        cursor = int(rng.integers(0, 20))
        src = int(rng.integers(0, 20))  # store rows of a session's runs are disjoint too
        while cursor < blocks_per * bs - 8 and src < cap - 1 and len(runs_o) < 40:
            n = int(rng.integers(1, 120))
            n = min(n, blocks_per * bs - cursor, cap - src)
            delta = int(rng.choice([0, int(rng.integers(-5000, 5000))]))
            r = {"session": s, "store_start": src, "len": n, "delta": delta}
            if rng.random() < 0.3:
                r["slots"] = O.slots(table, cursor, cursor + n, bs)
            else:
                r["block_table"], r["paged_start"] = table, cursor
            runs_o.append(r)
            cursor += n + int(rng.integers(0, 30))
            src += n + int(rng.integers(0, 30))

    stores = [[_rand((c, heads, 2 * d), dtype, g) for _ in range(layers)] for c in caps]
    kv = [_rand(SHAPES[layout](nblk, bs, heads, d), dtype, g) for _ in range(layers)]
    kv_d = [t.to(cuda) for t in kv]
    st_d = [[t.to(cuda) for t in per] for per in stores]
    inv = sk.inv_freq(rot, 1e6)
    k_scales = torch.tensor(rng.uniform(0.01, 0.1, layers), dtype=torch.float32)
    for r in runs_o:
        if "slots" in r:
            runs.append(RunSpec(r["session"], r["store_start"], r["len"], r["delta"],
                                slots=torch.from_numpy(r["slots"]).to(cuda)))
        else:
            runs.append(RunSpec(r["session"], r["store_start"], r["len"], r["delta"],
                                block_table=r["block_table"], paged_start=r["paged_start"]))

    prev = sk.set_load_kernel(kernel)
    try:
        la = Launcher(KVLayers(kv_d, bs, layout, fp8=dtype == O.E4M3))
        ptrs = np.array([[t.data_ptr() for t in per] for per in st_d], dtype=np.uint64)
        view = StoreView(ptrs, np.array(caps, np.int64), heads * 2 * d, 2 * d)
        la.load(runs, view, inv.to(cuda), k_scales=k_scales.to(cuda), check=True)
        torch.cuda.synchronize()
    finally:
        sk.set_load_kernel(prev)

    deltas = sorted({r["delta"] for r in runs_o if r["delta"]})
    tables = reference_tables(deltas, inv.numpy(), cuda) if deltas else None
    for r in runs_o:
        r["table"] = deltas.index(r["delta"]) if r["delta"] else -1
    paged = []
    for t in kv:
        geo = describe(t, bs, layout)
        paged.append(O.Paged(_bits(t).reshape(-1).copy(), 0, geo.v_offset, geo.blk_stride,
                             geo.off_stride, geo.head_stride, bs, heads, d))
    O.load([[_bits(t) for t in per] for per in stores], runs_o, paged, tables, dtype,
           k_scales.numpy())
    for li in range(layers):
        assert_cache_matches(_bits(kv_d[li]), paged[li], dtype, (seed, li))
        # the save below starts from what the load actually wrote (for e4m3 a
        # K code may sit one step from the oracle's)
        paged[li].flat = _bits(kv_d[li]).reshape(-1).copy()

    # and the save gathers the landed rows back out
    fresh = [[torch.zeros_like(t) for t in per] for per in st_d]
    fptrs = np.array([[t.data_ptr() for t in per] for per in fresh], dtype=np.uint64)
    fview = StoreView(fptrs, np.array(caps, np.int64), heads * 2 * d, 2 * d)
    la.save([RunSpec(r.session, r.store_start, r.length, slots=r.slots,
                     block_table=r.block_table, paged_start=r.paged_start) for r in runs],
            fview, check=True)
    torch.cuda.synchronize()
    out = [[np.zeros_like(_bits(t)) for t in per] for per in stores]
    O.save(out, runs_o, paged)
    for s in range(n_sessions):
        for li in range(layers):
            assert _bits(fresh[s][li]).tobytes() == out[s][li].tobytes(), (seed, s, li)
