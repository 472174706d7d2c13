"""GPU parity of the native shift kernels against the CPU oracle, through the C ABI.

Every case compares the bits the CUDA path writes with the bits the oracle
computes from the same inputs.  For bf16/fp16/fp32 K is re-rotated in fp32
with the reference's operation order and rounded once, so the comparison is
exact: V, every slot and every rotated K element must be bit-identical (which
is within the north-star bar of 1 bf16 ulp of the fp32 rotation).  For e4m3
the layer's K scale cancels and the kernel rounds once, so each K code is
within one e4m3 step of the oracle's (the north-star FP8 bar) and V is
identical.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from marathon_b200 import _lib
from marathon_b200 import shift_kernels as sk
from marathon_b200.paged import KVLayers
from marathon_b200.shift_kernels import Launcher, RunSpec, StoreView
from oracle import shift_oracle as O
from parity import assert_cache_matches, assert_k_codes_match, reference_tables

pytestmark = pytest.mark.gpu

DELTAS = [-3000, -4, 0, 4, 186, 10000]
H, D, BS = 8, 128, 16

TORCH_OF = {O.BF16: torch.bfloat16, O.F16: torch.float16, O.F32: torch.float32,
            O.E4M3: torch.float8_e4m3fn}


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def rand(shape, dtype: str, gen, scale=1.0):
    x = torch.randn(shape, generator=gen) * scale
    if dtype == O.E4M3:
        return x.clamp(-448, 448).to(torch.float8_e4m3fn)
    return x.to(TORCH_OF[dtype])


def fused_paged(kv_bits: np.ndarray, hnd: bool, heads=H, d=D, bs=BS) -> O.Paged:
    flat = kv_bits.reshape(-1).copy()
    if hnd:
        blk, head, off = heads * bs * 2 * d, bs * 2 * d, 2 * d
    else:
        blk, off, head = bs * heads * 2 * d, heads * 2 * d, 2 * d
    return O.Paged(flat, 0, d, blk, off, head, bs, heads, d)


def inv128():
    return sk.inv_freq(128, 1e6)


@pytest.fixture(params=["lsu", "bulk"])
def load_kernel(request, cuda):
    """Run a batched-load test through each load kernel (128-bit loads / TMA bulk).

    The process default ("auto") picks one of the two per dtype; forcing each
    covers both for every case.
    """
    prev = sk.set_load_kernel(request.param)
    yield request.param
    sk.set_load_kernel(prev)


# ------------------------------------------------------------------ tables
def test_rope_tables_are_the_references_gpu_tables(cuda, golden):
    """The table kernel reproduces the reference's tables as its GPU path builds
    them (torch fp32 cos/sin of ``float(delta) * inv_freq`` on the device) bit for
    bit, for rotary 128 and 64; and lies within one fp32 ulp of the correctly
    rounded values the oracle uses on the CPU."""
    deltas = golden["table_deltas"]
    for rot in (128, 64):
        inv = sk.inv_freq(rot, 1e6)
        got = sk.rope_tables(torch.tensor(deltas, device=cuda), inv.to(cuda)).cpu().numpy()
        assert np.array_equal(got, reference_tables(deltas, inv.numpy(), cuda)), rot
        exact = O.rope_tables(deltas, inv.numpy())
        assert O.ulp_distance(got, exact, O.F32).max() <= 1, rot


def test_rope_shift_fields_match_reference_structure(cuda, golden):
    for d in (-566, 0, 186):
        sh = sk.rope_shift(d, 128, inv128(), cuda)
        cos, sgn, partner = O.branchless_tables(sh.table.cpu().numpy(), 128)
        assert np.array_equal(sh.cos.cpu().numpy(), cos)
        assert np.array_equal(sh.sgn.cpu().numpy(), sgn)
        assert np.array_equal(sh.partner.cpu().numpy(), golden[f"tab_{d}_partner"])
        dist = O.ulp_distance(sh.emb_cos.cpu().numpy(), golden[f"tab_{d}_emb_cos"], O.F32)
        assert dist.max() <= 1


# ---------------------------------------------------- single-layer scatter
@pytest.mark.parametrize("delta", DELTAS)
@pytest.mark.parametrize("hnd", [True, False])
@pytest.mark.parametrize("n", [64, 37])
def test_scatter_shifted_bit_exact(cuda, delta, hnd, n):
    """Port of the reference's Triton-vs-torch test (test_shift_kernels.py:46-78), exact."""
    nblocks = 64
    g = torch.Generator().manual_seed(delta * 7 + n)
    src = rand((n, H, 2 * D), O.BF16, g)
    shape = (nblocks, H, BS, 2 * D) if hnd else (nblocks, BS, H, 2 * D)
    kv = rand(shape, O.BF16, g)
    table = torch.randperm(nblocks, generator=g)[: -(-n // BS) + 1]
    pos = torch.arange(3, 3 + n)
    slots = table[pos // BS] * BS + pos % BS
    shift = sk.rope_shift(delta, D, inv128(), cuda)
    got = kv.to(cuda)
    sk.scatter_shifted(src.to(cuda), got, slots.to(cuda), BS, hnd, shift, check=True)

    paged = fused_paged(bits(kv), hnd)
    tab = shift.table.cpu().numpy() if delta else None
    O.scatter_shifted(bits(src), paged, slots.numpy(), tab, O.BF16)
    assert np.array_equal(bits(got).reshape(-1), paged.flat)


def test_scatter_matches_reference_golden_vectors(cuda, golden):
    """Against the reference's own outputs: every K element within one bf16 ulp of
    its fp32 rotation (no allowance), V bit-exact."""
    src = torch.from_numpy(golden["bf16_src"].view(np.int16).copy()).view(torch.bfloat16)
    slots = torch.from_numpy(golden["bf16_slots"])
    for delta in DELTAS:
        for hnd in (True, False):
            shape = (64, H, BS, 2 * D) if hnd else (64, BS, H, 2 * D)
            kv = torch.zeros(shape, dtype=torch.bfloat16, device=cuda)
            sh = sk.rope_shift(delta, D, inv128(), cuda)
            sk.scatter_shifted(src.to(cuda), kv, slots.to(cuda), BS, hnd, sh, check=True)
            blk, off = slots // BS, slots % BS
            kc = kv.cpu()
            rows = kc[blk, :, off] if hnd else kc[blk, off]
            b = bits(rows)
            assert np.array_equal(b[..., D:], golden["bf16_src"][..., D:])
            # every K element within one bf16 ulp of the reference's fp32 rotation
            ok = O.within_one_step(b[..., :D], golden[f"f32r_k_{delta}"], O.BF16)
            assert ok.all(), (delta, hnd, int((~ok).sum()))
            assert O.ulp_distance(b[..., :D], golden[f"bf16_k_{delta}"], O.BF16).max() <= 1


@pytest.mark.parametrize("dtype", [O.F16, O.F32, O.E4M3])
@pytest.mark.parametrize("delta", [-566, 186])
def test_scatter_other_dtypes(cuda, dtype, delta):
    n, nblocks = 45, 16
    g = torch.Generator().manual_seed(abs(delta))
    scale = 20.0 if dtype == O.E4M3 else 1.0
    src = rand((n, H, 2 * D), dtype, g, scale)
    kv = rand((nblocks, BS, H, 2 * D), dtype, g, scale)
    slots = torch.randperm(nblocks * BS, generator=g)[:n].to(torch.int64)
    shift = sk.rope_shift(delta, D, inv128(), cuda)
    k_scale = torch.tensor([0.037], dtype=torch.float32)
    got = kv.to(cuda)
    sk.scatter_shifted(src.to(cuda), got, slots.to(cuda), BS, False, shift,
                       k_scale=k_scale.to(cuda), check=True)
    paged = fused_paged(bits(kv), False)
    O.scatter_shifted(bits(src), paged, slots.numpy(), shift.table.cpu().numpy(), dtype,
                      float(k_scale))
    assert_cache_matches(bits(got), paged, dtype, (dtype, delta))


def test_zero_length_load_is_a_noop(cuda):
    kv = torch.randn(4, 8, 16, 256, device=cuda).to(torch.bfloat16)
    before = kv.clone()
    src = torch.empty(0, 8, 256, dtype=torch.bfloat16, device=cuda)
    slots = torch.empty(0, dtype=torch.int64, device=cuda)
    sk.scatter_shifted(src, kv, slots, 16, True, sk.rope_shift(4, 128, inv128(), cuda))
    torch.cuda.synchronize()
    assert torch.equal(kv, before)


def test_cpu_tensors_are_refused_not_served():
    src = torch.zeros(4, 8, 256, dtype=torch.bfloat16)
    kv = torch.zeros(4, 16, 8, 256, dtype=torch.bfloat16)
    with pytest.raises(sk.ShiftError, match="no CPU path"):
        sk.scatter_shifted(src, kv, torch.arange(4), 16, False, None)


# ----------------------------------------------------------- batched paths
def _paged_shape(layout, nblk, bs, h, d):
    return {"nhd": (nblk, bs, h, 2 * d), "hnd": (nblk, h, bs, 2 * d),
            "split": (2, nblk, bs, h, d), "split_blocks": (nblk, 2, bs, h, d)}[layout]


def _oracle_paged(kv: torch.Tensor, layout: str, heads=H, d=D, bs=BS) -> O.Paged:
    from marathon_b200.paged import describe

    geo = describe(kv, bs, layout)
    return O.Paged(bits(kv).reshape(-1).copy(), 0, geo.v_offset, geo.blk_stride, geo.off_stride,
                   geo.head_stride, bs, heads, d)


def _batch_case(cuda, layout, dtype=O.BF16, heads=H, d=D, rot=None, layers=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    bs, nblk = BS, 48
    caps = [400, 260, 500]
    scale = 20.0 if dtype == O.E4M3 else 1.0
    stores = [[rand((c, heads, 2 * d), dtype, g, scale) for _ in range(layers)] for c in caps]
    kv = [rand(_paged_shape(layout, nblk, bs, heads, d), dtype, g, scale) for _ in range(layers)]
    perm = np.random.default_rng(seed).permutation(nblk).astype(np.int32)
    bt0, bt1, bt2 = perm[:14], perm[14:26], perm[26:40]
    slots2 = O.slots(bt2, 7, 7 + 97, bs)
    runs_o = [
        {"session": 0, "store_start": 3, "len": 190, "delta": 37, "block_table": bt0,
         "paged_start": 19},
        {"session": 1, "store_start": 250, "len": 9, "delta": -250, "block_table": bt1,
         "paged_start": 0},
        {"session": 2, "store_start": 401, "len": 97, "delta": 6759, "slots": slots2},
        {"session": 1, "store_start": 10, "len": 150, "delta": 0, "block_table": bt1,
         "paged_start": 30},
    ]
    return stores, kv, runs_o


def _run_batched_load(cuda, layout, dtype=O.BF16, heads=H, d=D, rotary=None, seed=0):
    rotary = rotary or d
    stores, kv, runs_o = _batch_case(cuda, layout, dtype, heads, d, seed=seed)
    layers = len(kv)
    stores_d = [[t.to(cuda) for t in per] for per in stores]
    kv_d = [t.to(cuda) for t in kv]
    inv = sk.inv_freq(rotary, 1e6)
    k_scales = torch.tensor([0.031, 0.07, 0.012][:layers], dtype=torch.float32)
    kl = KVLayers(kv_d, BS, layout, fp8=(dtype == O.E4M3))
    launcher = Launcher(kl)
    ptrs = np.array([[t.data_ptr() for t in per] for per in stores_d], dtype=np.uint64)
    view = StoreView(ptrs, np.array([t[0].shape[0] for t in stores], np.int64),
                     heads * 2 * d, 2 * d)
    runs = []
    for r in runs_o:
        if "slots" in r:
            runs.append(RunSpec(r["session"], r["store_start"], r["len"], r["delta"],
                                slots=torch.from_numpy(r["slots"]).to(cuda)))
        else:
            runs.append(RunSpec(r["session"], r["store_start"], r["len"], r["delta"],
                                block_table=r["block_table"], paged_start=r["paged_start"]))
    launcher.load(runs, view, inv.to(cuda), k_scales=k_scales.to(cuda), check=True)
    torch.cuda.synchronize()

    deltas = sorted({r["delta"] for r in runs_o if r["delta"]})
    tables = reference_tables(deltas, inv.numpy(), cuda)
    for r in runs_o:
        r["table"] = deltas.index(r["delta"]) if r["delta"] else -1
    st = [[bits(t) for t in per] for per in stores]
    paged = [_oracle_paged(t, layout, heads, d) for t in kv]
    O.load(st, runs_o, paged, tables, dtype, k_scales.numpy())
    for li in range(layers):
        assert_cache_matches(bits(kv_d[li]), paged[li], dtype, f"layer {li}")


@pytest.mark.parametrize("layout", ["nhd", "hnd", "split", "split_blocks"])
def test_batched_load_all_layouts_bit_exact(cuda, load_kernel, layout):
    _run_batched_load(cuda, layout)


@pytest.mark.parametrize("dtype", [O.F16, O.E4M3, O.F32])
def test_batched_load_dtypes(cuda, load_kernel, dtype):
    _run_batched_load(cuda, "nhd", dtype=dtype, seed=5)


@pytest.mark.parametrize("d,rotary", [(256, 64), (128, 64), (64, 64), (256, 256)])
def test_batched_load_head_geometries(cuda, load_kernel, d, rotary):
    _run_batched_load(cuda, "nhd", d=d, rotary=rotary, seed=d + rotary)


@pytest.mark.parametrize("dtype,d", [(O.F16, 64), (O.F16, 256), (O.E4M3, 256)])
def test_batched_load_other_dtype_head_sizes(cuda, load_kernel, dtype, d):
    """The remaining compiled (dtype, head_size) kernels, full rotary."""
    _run_batched_load(cuda, "nhd", dtype=dtype, d=d, seed=d + 7)


@pytest.mark.parametrize("heads", [1, 2, 4])
def test_batched_load_head_shards(cuda, load_kernel, heads):
    """The per-rank shapes of head-sharded tensor parallelism (8 heads over 8/4/2 ranks)."""
    _run_batched_load(cuda, "nhd", heads=heads, seed=heads)


@pytest.mark.parametrize("layout", ["nhd", "split"])
def test_batched_save_bit_exact_and_round_trip(cuda, layout):
    stores, kv, runs_o = _batch_case(cuda, layout, seed=9)
    layers = len(kv)
    kv_d = [t.to(cuda) for t in kv]
    fresh = [[torch.zeros(t[0].shape, dtype=torch.bfloat16, device=cuda) for _ in range(layers)]
             for t in stores]
    kl = KVLayers(kv_d, BS, layout)
    launcher = Launcher(kl)
    ptrs = np.array([[t.data_ptr() for t in per] for per in fresh], dtype=np.uint64)
    view = StoreView(ptrs, np.array([t[0].shape[0] for t in fresh], np.int64), H * 2 * D, 2 * D)
    runs = []
    for r in runs_o:
        if "slots" in r:
            runs.append(RunSpec(r["session"], r["store_start"], r["len"],
                                slots=torch.from_numpy(r["slots"]).to(cuda)))
        else:
            runs.append(RunSpec(r["session"], r["store_start"], r["len"],
                                block_table=r["block_table"], paged_start=r["paged_start"]))
    launcher.save(runs, view, check=True)
    torch.cuda.synchronize()
    ost = [[np.zeros(t[0].shape, dtype=np.uint16) for _ in range(layers)] for t in stores]
    paged = [_oracle_paged(t, layout) for t in kv]
    O.save(ost, runs_o, paged)
    for s in range(len(fresh)):
        for li in range(layers):
            assert np.array_equal(bits(fresh[s][li]), ost[s][li]), (s, li)
    # and a single layer out of the middle (the per-layer save_kv_layer shape)
    one = torch.zeros_like(fresh[0][1])
    v1 = StoreView(np.array([[one.data_ptr()]], dtype=np.uint64),
                   np.array([one.shape[0]], np.int64), H * 2 * D, 2 * D)
    launcher.save(runs[:1], v1, first_layer=1, n_layers=1, check=True)
    assert torch.equal(one, fresh[0][1])


def test_rejected_tokens_raise_without_fault_and_good_tokens_land(cuda, load_kernel):
    """Bad descriptors are flagged by the kernel (error word), never dereferenced."""
    g = torch.Generator().manual_seed(3)
    store = rand((64, H, 2 * D), O.BF16, g).to(cuda)
    kv = torch.zeros((8, BS, H, 2 * D), dtype=torch.bfloat16, device=cuda)
    launcher = Launcher(KVLayers([kv], BS, "nhd"))
    view = StoreView(np.array([[store.data_ptr()]], dtype=np.uint64),
                     np.array([64], np.int64), H * 2 * D, 2 * D)
    inv = inv128().to(cuda)
    # block 99 does not exist in an 8-block cache: tokens 16..31 of the run are refused
    bt = np.array([0, 99, 2], dtype=np.int32)
    with pytest.raises(sk.ShiftError, match="slot outside"):
        launcher.load([RunSpec(0, 0, 48, 5, block_table=bt, paged_start=0)], view, inv)
    torch.cuda.synchronize()
    assert kv[0].abs().sum() > 0 and kv[2].abs().sum() > 0
    # a run reading past the session buffer
    with pytest.raises(sk.ShiftError, match="store position"):
        launcher.load([RunSpec(0, 60, 16, 5, block_table=bt[:1], paged_start=0)], view, inv)
    # a session whose buffer is missing (address 0)
    v0 = StoreView(np.zeros((1, 1), dtype=np.uint64), np.array([64], np.int64), H * 2 * D, 2 * D)
    with pytest.raises(sk.ShiftError, match="session"):
        launcher.load([RunSpec(0, 0, 16, 5, block_table=bt[:1], paged_start=0)], v0, inv)
    # the context is still healthy
    launcher.load([RunSpec(0, 0, 16, 5, block_table=bt[:1], paged_start=0)], view, inv)
    torch.cuda.synchronize()


def test_native_status_codes_for_bad_arguments(cuda):
    lib = _lib.load()
    paged = _lib.Paged(1, 1, 1, 1, 16, 8, 100, _lib.BF16)  # head 100: not compiled
    rc = lib.mshift_scatter_shifted(1 << 20, 256, 256, 4, 1 << 20, 1 << 20, paged, 1 << 20,
                                    None, 100, None, 1 << 20, None)
    assert rc in (_lib.EINVAL, _lib.EUNSUPPORTED)
    assert lib.mshift_supported(_lib.BF16, 128, 128) == 1
    assert lib.mshift_supported(_lib.BF16, 100, 100) == 0


# -------------------------------------------------------- full-size checks
def _torch_reference_rows(store_rows: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """fp32 re-rotation in torch on the GPU: separate mul / mul / add kernels, no FMA."""
    d = store_rows.shape[-1] // 2
    h = table.shape[1]
    k = store_rows[..., :d].float()
    c, s = table[0], table[1]
    x, y = k[..., :h], k[..., h:]
    out = torch.cat((torch.sub(x * c, y * s), torch.add(y * c, x * s)), dim=-1)
    return torch.cat((out.to(store_rows.dtype), store_rows[..., d:]), dim=-1)


def _paged_rows(kv: torch.Tensor, layout: str, blk: torch.Tensor, off: torch.Tensor):
    """``[n, heads, 2D]`` rows of one layer's paged cache at (block, offset) pairs."""
    if layout == "nhd":
        return kv[blk, off]
    if layout == "hnd":
        return kv[blk, :, off]
    if layout == "split":
        return torch.cat((kv[0][blk, off], kv[1][blk, off]), dim=-1)
    return torch.cat((kv[blk, 0, off], kv[blk, 1, off]), dim=-1)  # split_blocks


def _reference_tables(deltas, inv_freq: torch.Tensor, on: str, device) -> dict:
    """The reference's tables (``shift_kernels.py:68-84``): torch's fp32 cos / sin of
    the fp32 angle ``float(delta) * inv_freq``, evaluated on ``on`` ("cpu", as its
    torch path and tests do, or "cuda", as its serving path does)."""
    inv = inv_freq.to(on, torch.float32)
    out = {}
    for d in deltas:
        ang = float(d) * inv
        emb = torch.cat((ang, ang))
        out[d] = (emb.cos().to(device), emb.sin().to(device))
    return out


def _ulp_bf16(r: torch.Tensor) -> torch.Tensor:
    """bf16 spacing at each fp32 value (2**(e-8) for |r| in [2**(e-1), 2**e))."""
    _, e = torch.frexp(r.abs())
    u = torch.ldexp(torch.ones_like(r), (e - 8).clamp(min=-133))
    return torch.where(r == 0, torch.full_like(r, 2.0**-133), torch.maximum(u, torch.full_like(r, 2.0**-133)))


def _check_north_star(wl, layout: str, tag) -> dict:
    """Every run x layer against the reference's fp32 rotation computed with the
    reference's own tables as its GPU path builds them (torch fp32 cos/sin on the
    device): V bit-exact, every K element within one bf16 ulp -- and in fact equal
    to the round-to-nearest of that rotation, since the tables and the arithmetic
    are the reference's.  Also counts, for information, the K elements more than
    one ulp from the rotation with the reference's CPU tables (torch's CPU cos/sin
    differ from the GPU's by an ulp here and there, which a cancelling sum can
    magnify)."""
    cfg = wl.cfg
    deltas = sorted({r.delta for r in wl.runs if r.delta})
    device = wl.kv[0].device
    gpu_tabs = _reference_tables(deltas, wl.inv_freq, "cuda", device)
    cpu_tabs = _reference_tables(deltas, wl.inv_freq, "cpu", device)
    stats = {"not_rne_gpu_tables": 0, "beyond_1ulp_cpu_tables": 0, "k_elements": 0}
    for li in range(cfg.layers):
        for r in wl.runs:
            rows = wl.stores[r.session][li][r.store_start : r.store_start + r.length]
            bt = wl.block_tables[r.session].long()
            pos = torch.arange(r.paged_start, r.paged_start + r.length, device=device)
            got = _paged_rows(wl.kv[li], layout, bt[pos // cfg.block_size],
                              pos % cfg.block_size)
            assert torch.equal(got[..., D:].view(torch.int16),
                               rows[..., D:].view(torch.int16)), (tag, li, r)
            if not r.delta:
                assert torch.equal(got.view(torch.int16), rows.view(torch.int16))
                continue
            kf = rows[..., :D].float()
            rot = torch.cat((-kf[..., D // 2 :], kf[..., : D // 2]), dim=-1)
            gk = got[..., :D].float()
            cos, sin = gpu_tabs[r.delta]
            ref = kf * cos + rot * sin  # the reference's torch path, in fp32
            bad = int(((gk - ref).abs() > _ulp_bf16(ref)).sum())
            assert bad == 0, (tag, li, r.delta, bad)
            stats["not_rne_gpu_tables"] += int((got[..., :D] != ref.to(torch.bfloat16)).sum())
            cos, sin = cpu_tabs[r.delta]
            ref = kf * cos + rot * sin
            stats["beyond_1ulp_cpu_tables"] += int(((gk - ref).abs() > _ulp_bf16(ref)).sum())
            stats["k_elements"] += gk.numel()
    return stats


def _check_workload_vs_torch(wl, layout: str, tag) -> None:
    """Every run x layer of a loaded workload against torch fp32 on the same GPU."""
    cfg = wl.cfg
    deltas = sorted({r.delta for r in wl.runs if r.delta})
    tables = sk.rope_tables(torch.tensor(deltas, device=wl.kv[0].device), wl.inv_freq)
    for li in range(cfg.layers):
        for r in wl.runs:
            rows = wl.stores[r.session][li][r.store_start : r.store_start + r.length]
            want = _torch_reference_rows(rows, tables[deltas.index(r.delta)]) if r.delta else rows
            bt = wl.block_tables[r.session].long()
            pos = torch.arange(r.paged_start, r.paged_start + r.length, device=rows.device)
            blk = bt[pos // cfg.block_size]
            off = pos % cfg.block_size
            got = _paged_rows(wl.kv[li], layout, blk, off)
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (tag, li, r)


@pytest.mark.parametrize("name", ["c0", "c0z", "c1", "c2"])
def test_baseline_configs_full_size_vs_torch_fp32(cuda, load_kernel, name):
    """Every layer of configs c0-c2 at full size: bit-exact against torch fp32 on the
    same GPU with the kernel's tables, and within the north-star bar (one bf16 ulp,
    V exact) of the reference's rotation with the reference's own tables."""
    from marathon_b200.workloads import build, config

    cfg = config(name)
    wl = build(cfg, cuda)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, "nhd"))
    launcher.load(wl.runs, wl.store_view(), wl.inv_freq, check=True)
    torch.cuda.synchronize()
    _check_workload_vs_torch(wl, "nhd", name)
    stats = _check_north_star(wl, "nhd", name)
    print(f"{name}: north-star check {stats}")
    assert stats["not_rne_gpu_tables"] == 0
    del wl
    torch.cuda.empty_cache()


@pytest.mark.parametrize("layout", ["hnd", "split", "split_blocks"])
def test_c1_full_segments_other_layouts_vs_torch_fp32(cuda, load_kernel, layout):
    """c1's three full-length segments (2 of 36 layers) in the non-default layouts."""
    from marathon_b200.workloads import build, config, scaled

    cfg = scaled(config("c1"), layers=2)
    wl = build(cfg, cuda, layout=layout)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, layout))
    launcher.load(wl.runs, wl.store_view(), wl.inv_freq, check=True)
    torch.cuda.synchronize()
    _check_workload_vs_torch(wl, layout, layout)
    del wl
    torch.cuda.empty_cache()


@pytest.mark.parametrize("lo,hi", [(3, 4), (4, 8)])
def test_c4_sessions_head_shard_vs_torch_fp32(cuda, load_kernel, lo, hi):
    """c4's 64 sessions (2 of 36 layers) as one tensor-parallel rank sees them:
    heads [lo, hi) of 8, every session's segments in one launch."""
    from marathon_b200.workloads import build, config, scaled

    cfg = scaled(config("c4"), layers=2)
    wl = build(cfg, cuda, head_lo=lo, head_hi=hi)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, "nhd"))
    launcher.load(wl.runs, wl.store_view(), wl.inv_freq, check=True)
    torch.cuda.synchronize()
    assert len(wl.runs) > 64
    _check_workload_vs_torch(wl, "nhd", (lo, hi))
    del wl
    torch.cuda.empty_cache()


def test_c2_two_layers_vs_numpy_oracle(cuda):
    """c2's full 28,608-token segment through the numpy oracle (2 of 40 layers)."""
    from marathon_b200.workloads import build, config, scaled

    cfg = scaled(config("c2"), layers=2)
    wl = build(cfg, cuda)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, "nhd"))
    launcher.load(wl.runs, wl.store_view(), wl.inv_freq, check=True)
    torch.cuda.synchronize()
    r = wl.runs[0]
    tables = reference_tables([r.delta], wl.inv_freq.cpu().numpy(), cuda)
    sl = O.slots(wl.block_tables_host[0], r.paged_start, r.paged_start + r.length, BS)
    for li in range(2):
        rows = bits(wl.stores[0][li][r.store_start : r.store_start + r.length])
        want_k = O.shift_k_bits(rows[..., :D], tables[0], O.BF16)
        got = bits(wl.kv[li]).reshape(-1, BS, H, 2 * D)
        g = got[sl // BS, sl % BS]
        assert np.array_equal(g[..., :D], want_k)
        assert np.array_equal(g[..., D:], rows[..., D:])


def test_c3_fp8_full_segment_vs_oracle(cuda, load_kernel):
    """c3 (e4m3, per-layer scales): 2 layers of the full segment through the oracle."""
    from marathon_b200.workloads import build, config, scaled

    cfg = scaled(config("c3"), layers=2)
    wl = build(cfg, cuda)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, "nhd", fp8=True))
    launcher.load(wl.runs, wl.store_view(), wl.inv_freq, k_scales=wl.k_scales, check=True)
    torch.cuda.synchronize()
    r = wl.runs[0]
    tables = reference_tables([r.delta], wl.inv_freq.cpu().numpy(), cuda)
    sl = O.slots(wl.block_tables_host[0], r.paged_start, r.paged_start + r.length, BS)
    ks = wl.k_scales.cpu().numpy()
    for li in range(2):
        rows = bits(wl.stores[0][li][r.store_start : r.store_start + r.length])
        want_k = O.shift_k_bits(rows[..., :D], tables[0], O.E4M3, float(ks[li]))
        got = bits(wl.kv[li]).reshape(-1, BS, H, 2 * D)[sl // BS, sl % BS]
        assert np.array_equal(got[..., D:], rows[..., D:])
        assert_k_codes_match(got[..., :D], want_k, O.E4M3, li)


def _oracle_layer_e4m3(args):
    rows, got, table, scale = args
    want = O.shift_k_bits(rows[..., :D], table, O.E4M3, scale)
    v_ok = np.array_equal(got[..., D:], rows[..., D:])
    steps = O.ulp_distance(got[..., :D], want, O.E4M3)
    return v_ok, int(steps.max()), int((steps > 0).sum())


def test_c3_fp8_every_layer_vs_oracle(cuda):
    """c3 (e4m3, per-layer scales), all 40 layers of the full segment, against the
    numpy oracle's dequantise -> rotate -> requantise: V bit-exact, every K code
    within one e4m3 step of the oracle's."""
    from concurrent.futures import ThreadPoolExecutor

    from marathon_b200.workloads import build, config

    cfg = config("c3")
    wl = build(cfg, cuda)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, "nhd", fp8=True))
    launcher.load(wl.runs, wl.store_view(), wl.inv_freq, k_scales=wl.k_scales, check=True)
    torch.cuda.synchronize()
    r = wl.runs[0]
    table = reference_tables([r.delta], wl.inv_freq.cpu().numpy(), cuda)[0]
    bt = wl.block_tables[0].long()
    pos = torch.arange(r.paged_start, r.paged_start + r.length, device=cuda)
    blk, off = bt[pos // BS], pos % BS
    ks = wl.k_scales.cpu().numpy()

    def layer(li):
        rows = bits(wl.stores[0][li][r.store_start : r.store_start + r.length])
        return rows, bits(wl.kv[li][blk, off]), table, float(ks[li])

    differ = 0
    with ThreadPoolExecutor(4) as pool:
        for li, (v_ok, worst, n_diff) in enumerate(pool.map(_oracle_layer_e4m3,
                                                            map(layer, range(cfg.layers)))):
            assert v_ok, li
            assert worst <= 1, (li, worst)
            differ += n_diff
    total = cfg.layers * r.length * H * D
    print(f"c3: {differ} of {total} K codes one step from the oracle's")
    assert differ <= total * 1e-4
    del wl
    torch.cuda.empty_cache()


def test_c4_one_head_shard_every_layer(cuda):
    """c4's 64 sessions as the last rank at TP8 holds them (one KV head), all 36
    layers in one launch: bit-exact against torch fp32 with the kernel's tables, and
    within the north-star bar of the reference's rotation with its own tables."""
    from marathon_b200.workloads import build, config

    cfg = config("c4")
    wl = build(cfg, cuda, head_lo=7, head_hi=8)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, "nhd"))
    launcher.load(wl.runs, wl.store_view(), wl.inv_freq, check=True)
    torch.cuda.synchronize()
    assert cfg.layers == 36 and len(wl.runs) > 64
    _check_workload_vs_torch(wl, "nhd", "c4 head 7")
    stats = _check_north_star(wl, "nhd", "c4 head 7")
    print(f"c4 head 7: north-star check {stats}")
    assert stats["not_rne_gpu_tables"] == 0
    del wl
    torch.cuda.empty_cache()


def test_shift_round_trip_property_full_size(cuda):
    """Load by +delta, save, load by -delta: V bit-exact, K back within bf16 rounding."""
    from marathon_b200.workloads import build, config, scaled

    cfg = scaled(config("c2"), layers=4)
    wl = build(cfg, cuda)
    launcher = Launcher(KVLayers(wl.kv, cfg.block_size, "nhd"))
    view = wl.store_view()
    launcher.load(wl.runs, view, wl.inv_freq, check=True)
    r = wl.runs[0]
    cap = r.paged_start + r.length  # rows land at their new positions
    back = [torch.zeros((cap, *t.shape[1:]), dtype=t.dtype, device=cuda) for t in wl.stores[0]]
    bview = StoreView(np.array([[t.data_ptr() for t in back]], dtype=np.uint64),
                      np.array([back[0].shape[0]], np.int64), view.st_tok, view.st_head)
    launcher.save([RunSpec(0, r.paged_start, r.length, block_table=wl.block_tables[0],
                           paged_start=r.paged_start)], bview, check=True)
    # rows now sit at store positions [paged_start, +len) in the new coordinates
    for t in wl.kv:
        t.zero_()
    launcher.load([RunSpec(0, r.paged_start, r.length, -r.delta, block_table=wl.block_tables[0],
                           paged_start=r.store_start)], bview, wl.inv_freq, check=True)
    torch.cuda.synchronize()
    pos = torch.arange(r.store_start, r.store_start + r.length, device=cuda)
    bt = wl.block_tables[0].long()
    for li in range(4):
        got = wl.kv[li][bt[pos // BS], pos % BS]
        orig = wl.stores[0][li][r.store_start : r.store_start + r.length]
        assert torch.equal(got[..., D:].view(torch.int16), orig[..., D:].view(torch.int16))
        # two bf16 roundings, each at most 2^-9 of the rotated pair's magnitude, come
        # back through a rotation: bound the error by the RoPE pair (i, i + D/2)
        k1, k0 = got[..., :D].float(), orig[..., :D].float()
        pair = k0[..., : D // 2].abs() + k0[..., D // 2 :].abs()
        bound = 2.0**-7 * torch.cat((pair, pair), dim=-1)
        assert bool(((k1 - k0).abs() <= bound).all())
