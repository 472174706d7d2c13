"""``torch.ops.marathon.*``: the operator-registry face of the shift path.

CPU: the operators are registered with their schemas and refuse CPU tensors
(there is no CPU implementation).  GPU: each operator lands the same bits as
the oracle / the launcher path on the same inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import marathon_b200  # noqa: F401  (registers the operators)
from marathon_b200 import shift_kernels as sk
from marathon_b200.shift_kernels import ShiftError
from oracle import shift_oracle as O
from parity import reference_tables

H, D, BS = 8, 128, 16


def test_operators_are_registered_with_their_schemas():
    ops = torch.ops.marathon
    assert "Tensor(a1!)[] kv" in str(ops.shift_load.default._schema)
    assert "Tensor(a1!)[] stores" in str(ops.shift_save.default._schema)
    assert "Tensor(a1!) kv" in str(ops.scatter_shifted.default._schema)


def test_operators_refuse_cpu_tensors():
    kv = torch.zeros(4, BS, H, 2 * D, dtype=torch.bfloat16)
    src = torch.zeros(3, H, 2 * D, dtype=torch.bfloat16)
    with pytest.raises(ShiftError, match="CUDA"):
        torch.ops.marathon.scatter_shifted(src, kv, torch.arange(3), BS, False, None)
    seg = torch.tensor([[0, 0, 0, 3, 5]])
    with pytest.raises(ShiftError, match="CUDA"):
        torch.ops.marathon.shift_load([src], [kv], seg, [torch.arange(4, dtype=torch.int32)],
                                      sk.inv_freq(D, 1e6), BS, "nhd", None)


def _case(cuda, seed=0, layers=3):
    g = torch.Generator().manual_seed(seed)
    caps = [300, 220]
    stores = [[(torch.randn(c, H, 2 * D, generator=g)).to(torch.bfloat16) for _ in range(layers)]
              for c in caps]
    kv = [torch.randn(40, BS, H, 2 * D, generator=g).to(torch.bfloat16) for _ in range(layers)]
    perm = np.random.default_rng(seed).permutation(40).astype(np.int32)
    tables = [perm[:20], perm[20:40]]
    # (session, src_start, dst_start, length, delta)
    seg = [(0, 5, 12, 150, 7), (1, 100, 64, 90, -36), (0, 200, 200, 60, 0)]
    return stores, kv, tables, seg


@pytest.mark.gpu
def test_shift_load_operator_matches_the_oracle(cuda):
    stores, kv, tables, seg = _case(cuda)
    inv = sk.inv_freq(D, 1e6)
    st_d = [t.to(cuda) for per in stores for t in per]
    kv_d = [t.to(cuda) for t in kv]
    bt_d = [torch.from_numpy(t).to(cuda) for t in tables]
    torch.ops.marathon.shift_load(st_d, kv_d, torch.tensor(seg), bt_d, inv.to(cuda), BS, "nhd",
                                  None)
    torch.cuda.synchronize()
    deltas = sorted({s[4] for s in seg if s[4]})
    tabs = reference_tables(deltas, inv.numpy(), cuda)
    runs = [{"session": s, "store_start": a, "len": n, "paged_start": b,
             "block_table": tables[s], "table": deltas.index(d) if d else -1}
            for s, a, b, n, d in seg]
    st = [[t.view(torch.int16).numpy().view(np.uint16) for t in per] for per in stores]
    blk, off, head = BS * H * 2 * D, H * 2 * D, 2 * D
    paged = [O.Paged(t.view(torch.int16).numpy().view(np.uint16).reshape(-1).copy(), 0, D, blk,
                     off, head, BS, H, D) for t in kv]
    O.load(st, runs, paged, tabs, O.BF16, None)
    for li, t in enumerate(kv_d):
        got = t.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1)
        assert np.array_equal(got, paged[li].flat), li


@pytest.mark.gpu
def test_shift_save_operator_round_trips(cuda):
    stores, kv, tables, seg = _case(cuda, seed=3)
    kv_d = [t.to(cuda) for t in kv]
    fresh = [torch.zeros_like(t).to(cuda) for per in stores for t in per]
    bt_d = [torch.from_numpy(t).to(cuda) for t in tables]
    save = torch.tensor([(s, 0, b, n, 0) for s, _, b, n, _ in seg])
    torch.ops.marathon.shift_save(kv_d, fresh, save, bt_d, BS, "nhd")
    torch.cuda.synchronize()
    L = len(kv)
    for s, _, b, n, _ in seg:
        pos = torch.arange(b, b + n)
        blk = torch.from_numpy(tables[s]).long()[pos // BS]
        for li in range(L):
            want = kv[li][blk, pos % BS]
            got = fresh[s * L + li][b : b + n].cpu()
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (s, li)


@pytest.mark.gpu
def test_scatter_shifted_operator_matches_the_function(cuda):
    stores, kv, tables, _ = _case(cuda, seed=5, layers=1)
    inv = sk.inv_freq(D, 1e6).to(cuda)
    shift = sk.rope_shift(186, D, inv, cuda)
    src = stores[0][0][:100].to(cuda)
    slots = torch.from_numpy(O.slots(tables[0], 3, 103, BS)).to(cuda)
    a, b = kv[0].to(cuda), kv[0].to(cuda)
    torch.ops.marathon.scatter_shifted(src, a, slots, BS, False, shift.table)
    sk.scatter_shifted(src, b, slots, BS, False, shift)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert not torch.equal(a.view(torch.int16), kv[0].to(cuda).view(torch.int16))


@pytest.mark.gpu
def test_operators_trace_under_torch_compile(cuda):
    """Dynamo traces through the operators (their fake implementations) and the
    compiled call mutates the caches exactly as the eager call does."""
    stores, kv, tables, seg = _case(cuda, seed=7)
    inv = sk.inv_freq(D, 1e6).to(cuda)
    st_d = [t.to(cuda) for per in stores for t in per]
    bt_d = [torch.from_numpy(t).to(cuda) for t in tables]
    segs = torch.tensor(seg)
    a = [t.to(cuda) for t in kv]
    b = [t.to(cuda) for t in kv]

    def step(caches):
        torch.ops.marathon.shift_load(st_d, caches, segs, bt_d, inv, BS, "nhd", None)

    torch.compile(step, backend="eager", fullgraph=True)(a)
    step(b)
    torch.cuda.synchronize()
    for x, y in zip(a, b, strict=True):
        assert torch.equal(x.view(torch.int16), y.view(torch.int16))
